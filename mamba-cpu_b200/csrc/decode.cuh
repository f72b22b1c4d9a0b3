// decode.cuh -- single-step (decode) launchers: selective_state_update and causal_conv1d_update.
#pragma once

#include "common.cuh"

namespace mb200 {

cudaError_t launch_state_update(const mb200_state_update_params& p, cudaStream_t stream);
cudaError_t launch_conv_update(const mb200_conv1d_update_params& p, cudaStream_t stream);

}  // namespace mb200
