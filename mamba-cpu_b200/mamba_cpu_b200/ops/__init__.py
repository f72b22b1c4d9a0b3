from mamba_cpu_b200.ops.causal_conv1d import causal_conv1d_fn, causal_conv1d_update
from mamba_cpu_b200.ops.selective_scan_interface import selective_scan_fn
from mamba_cpu_b200.ops.selective_state_update import selective_state_update
from mamba_cpu_b200.ops.ssd_combined import mamba_chunk_scan_combined

__all__ = [
    "causal_conv1d_fn",
    "causal_conv1d_update",
    "mamba_chunk_scan_combined",
    "selective_scan_fn",
    "selective_state_update",
]
