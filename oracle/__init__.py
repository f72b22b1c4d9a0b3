"""CPU checkers for the CUDA selective scan and causal conv1d. TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) import this package. The product (``mamba_cpu_b200``) never does.

Two checkers live here:

* :mod:`oracle.f64` -- a float64 restatement in plain C (``oracle.c``) of the reference's
  selective-scan forward/backward (mamba-cpu ``csrc/selective_scan.cpp:120-145, 168-248``),
  its conv1d (``src/mamba_cpu/ops/causal_conv1d.py:16-85``) and decode step
  (``src/mamba_cpu/ops/selective_state_update.py:5-57``).
* :mod:`oracle.ref_c` -- the reference's OWN C++ kernel, compiled from its sources by
  ``oracle/Makefile`` into ``oracle/_ref/`` and exposed with the same Python-level interface as
  the reference's nanobind module ``mamba_cpu._C`` (``csrc/bindings.cpp:18-85``).
"""

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_F64 = os.path.join(HERE, "_build", "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libmamba_cpu_ref.so")
# The reference checkout: $MAMBA_REF_DIR, else a directory named `reference` beside this
# repository's checkout.
REF_DIR = os.environ.get("MAMBA_REF_DIR", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def build(ref: bool = True) -> None:
    """Compile the float64 oracle, and the reference kernel when its sources are present."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(os.path.join(REF_DIR, "csrc")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_DIR={REF_DIR}"], check=True)


def ensure_f64() -> str:
    if not os.path.exists(LIB_F64):
        build(ref=False)
    return LIB_F64


def ref_available() -> bool:
    return os.path.exists(LIB_REF)
