"""B200-native (sm_100a) Mamba-1 selective scan and causal conv1d.

The public functions have the signatures of mamba-cpu / mamba_ssm / causal_conv1d
(mamba-cpu src/mamba_cpu/__init__.py:3-23) and run hand-written CUDA kernels from
libmamba_b200.so on CUDA tensors. Non-CUDA tensors are rejected, as the reference rejects
non-CPU ones. ``mamba_chunk_scan_combined`` adds the Mamba-2 SSD scan forward (a roadmap item of
the reference) with upstream mamba_ssm's signature. ``selective_scan_ref`` and ``causal_conv1d_ref`` are plain PyTorch versions of the
two operators (any device), exported as the reference exports its own.
"""

from mamba_cpu_b200 import hf, parallel
from mamba_cpu_b200.ops import (
    causal_conv1d_fn,
    causal_conv1d_update,
    mamba_chunk_scan_combined,
    selective_scan_fn,
    selective_state_update,
)
from mamba_cpu_b200.reference import causal_conv1d_ref, selective_scan_ref

__version__ = "0.1.0"

__all__ = [
    "causal_conv1d_fn",
    "causal_conv1d_ref",
    "causal_conv1d_update",
    "hf",
    "mamba_chunk_scan_combined",
    "parallel",
    "selective_scan_fn",
    "selective_scan_ref",
    "selective_state_update",
]
