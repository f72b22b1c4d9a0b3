// peer.cu -- one-shot sum of a float buffer over the GPUs of a node, through peer memory.
//
// Used for the dB / dC partial sums of a channel-sharded backward (one exchange per call,
// ~0.5 MB at BASELINE config 2). Every rank owns an exchange buffer of two slots of n floats and
// a signal pad of `world` uint32 words, mapped into the other ranks' address spaces with CUDA IPC
// (plain peer mappings over NVLink; no multicast objects, no bulk or TMA loads from peers).
//
// One call = one kernel (peer_allreduce) of MB200_PEER_BLOCKS CTAs. Element i of the exchange
// [a | b] belongs to the same CTA j on every rank (the grid and the index mapping do not depend
// on the rank), so the CTAs synchronise pairwise and never grid-wide:
//   * CTA j copies its elements into this rank's slot (e & 1), where e is CTA j's call number
//     (a per-CTA counter in device memory), then stores e into word (rank, j) of every rank's
//     signal pad (release, system scope);
//   * it waits until words (q, j) of its own pad reached e for every rank q (acquire, bounded),
//     then writes the rank-ordered sum of its elements of all slots back to a | b -- the same
//     bits on every rank.
// CTA j of a rank reuses a slot two calls later; by then CTA j of every other rank has
// signalled the call in between, which it does only after its reads of the slot (the previous
// kernel) completed, so one signal per CTA and call suffices. The counters live in device
// memory, so the call is valid inside CUDA graphs.
// A CTA whose wait for another rank runs out does not sum (the other rank's slot may not hold
// this call's partials yet): it fills its elements of a | b with NaN, sets fault bit 1 and the
// sticky word counters[MB200_PEER_BLOCKS], which the host reads to refuse the poisoned result.
// The signals stay in step (every CTA still signals every call), so a rank that arrives late
// completes its own call with a correct sum.
#include <cuda_runtime.h>
#include <string.h>

#include "common.cuh"
#include "mamba_b200.h"
#include "stage.cuh"

namespace mb200 {

namespace {

constexpr int kFaultPeerTimeout = 2;
constexpr int kPeerThreads = 256;
constexpr int kMaxUnrolledRanks = 8;
constexpr int64_t kDefaultTimeoutUs = 30ll * 1000 * 1000;  // a rank may lag (e.g. checkpointing)

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Nanoseconds since an arbitrary origin (the GPU's global timer).
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float4 add4(float4 x, float4 y) {
  return make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
}

// Quad i (elements 4i .. 4i+3) of the concatenation [a (na) | b (nb)]; elements past na + nb read
// as 0 and are not written. `vec`: a and b are 16-byte aligned and na, nb multiples of 4.
__device__ __forceinline__ float4 load_quad(const float* a, int64_t na, const float* b, int64_t nb, bool vec,
                                            int64_t i) {
  if (vec) return 4 * i < na ? reinterpret_cast<const float4*>(a)[i] : reinterpret_cast<const float4*>(b)[i - na / 4];
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t x = 4 * i + k;
    v[k] = x < na ? a[x] : x < na + nb ? b[x - na] : 0.f;
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

__device__ __forceinline__ void store_quad(float* a, int64_t na, float* b, int64_t nb, bool vec, int64_t i,
                                           float4 q) {
  if (vec) {
    if (4 * i < na)
      reinterpret_cast<float4*>(a)[i] = q;
    else
      reinterpret_cast<float4*>(b)[i - na / 4] = q;
    return;
  }
  const float v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t x = 4 * i + k;
    if (x < na)
      a[x] = v[k];
    else if (x < na + nb)
      b[x - na] = v[k];
  }
}

// Both passes over this thread's quads of the exchange (slot quads nq = ceil((na + nb) / 4)).
// kSum = false copies [a | b] into this rank's slot at quad `off`; kSum = true writes the
// rank-ordered sum of all slots back to [a | b]. Quad i is handled by the same CTA on every rank
// (the mapping depends only on the grid and nq) and by the same thread in both passes, so the
// sum may overwrite its own source.
template <bool kSum>
__device__ __forceinline__ void exchange_pass(float* a, int64_t na, float* b, int64_t nb, bool vec,
                                              float* const* bufs, int64_t off, int rank, int world) {
  const int64_t nq = (na + nb + 3) / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += stride) {
    if (!kSum) {
      reinterpret_cast<float4*>(bufs[rank])[off + i] = load_quad(a, na, b, nb, vec, i);
      continue;
    }
    float4 acc;
    if (world <= kMaxUnrolledRanks) {
      float4 v[kMaxUnrolledRanks];
#pragma unroll
      for (int q = 0; q < kMaxUnrolledRanks; ++q)  // every load in flight before the first add
        if (q < world) v[q] = __ldcv(reinterpret_cast<const float4*>(bufs[q]) + off + i);
      acc = v[0];
#pragma unroll
      for (int q = 1; q < kMaxUnrolledRanks; ++q)
        if (q < world) acc = add4(acc, v[q]);
    } else {
      acc = __ldcv(reinterpret_cast<const float4*>(bufs[0]) + off + i);
      for (int q = 1; q < world; ++q) acc = add4(acc, __ldcv(reinterpret_cast<const float4*>(bufs[q]) + off + i));
    }
    store_quad(a, na, b, nb, vec, i, acc);
  }
}

// Fills this CTA's quads of [a | b] with NaN (the result of a call whose wait ran out).
__device__ __forceinline__ void poison_pass(float* a, int64_t na, float* b, int64_t nb, bool vec) {
  const int64_t nq = (na + nb + 3) / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float q = __int_as_float(0x7fc00000);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += stride)
    store_quad(a, na, b, nb, vec, i, make_float4(q, q, q, q));
}

__global__ void __launch_bounds__(kPeerThreads) peer_allreduce(float* a, int64_t na, float* b, int64_t nb,
                                                               float* const* bufs, uint32_t* const* pads,
                                                               uint32_t* counters, int rank, int world,
                                                               uint64_t timeout_ns) {
  __shared__ uint32_t s_e;
  __shared__ int s_late;
  const int j = blockIdx.x;
  if (threadIdx.x == 0) {
    s_e = counters[j] + 1u;  // only CTA j of this rank's calls touches counters[j]
    counters[j] = s_e;
    s_late = 0;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int64_t off = (int64_t)(e & 1u) * ((na + nb + 3) / 4);  // slot, in quads
  const bool vec = aligned16(a) && aligned16(b) && na % 4 == 0 && nb % 4 == 0;  // source access only
  exchange_pass<false>(a, na, b, nb, vec, bufs, off, rank, world);
  __syncthreads();
  if (threadIdx.x < world) {
    __threadfence_system();  // the CTA's copies (ordered before by the barrier), then the signal
    st_release_sys(pads[threadIdx.x] + rank * MB200_PEER_BLOCKS + j, e);
    const uint32_t* word = pads[rank] + threadIdx.x * MB200_PEER_BLOCKS + j;
    // Bounded wait: timeout_ns of global time, or (should the timer not advance) timeout_ns / 64
    // polls, each of which takes far longer than 64 ns (a system-scope load and a sleep).
    const uint64_t t0 = global_ns();
    for (uint64_t it = 1; (int)(ld_acquire_sys(word) - e) < 0; ++it) {
      if (((it & 255) == 0 && global_ns() - t0 > timeout_ns) || it > timeout_ns / 64) {
        atomicOr(&g_mb200_fault, kFaultPeerTimeout);
        atomicOr(&counters[MB200_PEER_BLOCKS], 1u);  // sticky: the host refuses this result
        s_late = 1;
        break;
      }
      __nanosleep(100);
    }
  }
  __syncthreads();
  if (s_late)
    poison_pass(a, na, b, nb, vec);
  else
    exchange_pass<true>(a, na, b, nb, vec, bufs, off, rank, world);
}

}  // namespace

cudaError_t read_fault_peer(int* out) { return read_fault_word(out); }

}  // namespace mb200

using namespace mb200;

extern "C" {

MB200_API int mb200_ipc_handle(void* dev_ptr, unsigned char handle[MB200_IPC_HANDLE_BYTES]) {
  if (dev_ptr == nullptr || handle == nullptr) return MB200_ERR_NULL_POINTER;
  static_assert(sizeof(cudaIpcMemHandle_t) == MB200_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, dev_ptr) != cudaSuccess) return MB200_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return MB200_OK;
}

MB200_API int mb200_ipc_open(const unsigned char handle[MB200_IPC_HANDLE_BYTES], void** dev_ptr) {
  if (dev_ptr == nullptr || handle == nullptr) return MB200_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MB200_ERR_CUDA;
  return MB200_OK;
}

MB200_API int mb200_peer_alloc(size_t bytes, void** dev_ptr) {
  if (dev_ptr == nullptr) return MB200_ERR_NULL_POINTER;
  if (cudaMalloc(dev_ptr, bytes) != cudaSuccess) return MB200_ERR_CUDA;
  if (cudaMemset(*dev_ptr, 0, bytes) != cudaSuccess) return MB200_ERR_CUDA;
  return MB200_OK;
}

MB200_API int mb200_peer_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return MB200_ERR_NULL_POINTER;
  return cudaFree(dev_ptr) == cudaSuccess ? MB200_OK : MB200_ERR_CUDA;
}

MB200_API int mb200_ipc_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return MB200_ERR_NULL_POINTER;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? MB200_OK : MB200_ERR_CUDA;
}

MB200_API int mb200_peer_sum_f32(float* a, int64_t na, float* b, int64_t nb, float* const* peer_bufs,
                                 uint32_t* const* peer_pads, uint32_t* counters, int rank, int world,
                                 int64_t timeout_us, void* stream) {
  reset_launches();
  if ((a == nullptr && na > 0) || (b == nullptr && nb > 0) || peer_bufs == nullptr || peer_pads == nullptr ||
      counters == nullptr)
    return MB200_ERR_NULL_POINTER;
  if (na < 0 || nb < 0 || world < 1 || world > kPeerThreads || rank < 0 || rank >= world) return MB200_ERR_BAD_SHAPE;
  if (na + nb == 0) return MB200_OK;
  peer_allreduce<<<MB200_PEER_BLOCKS, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      a, na, b, nb, peer_bufs, peer_pads, counters, rank, world,
      static_cast<uint64_t>(timeout_us > 0 ? timeout_us : kDefaultTimeoutUs) * 1000ull);
  if (cudaGetLastError() != cudaSuccess) return MB200_ERR_CUDA;
  note_launches(1);
  return MB200_OK;
}

}  // extern "C"
