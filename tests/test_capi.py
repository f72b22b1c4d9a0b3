"""The C ABI (include/mamba_b200.h) without a GPU: the library loads, exports every declared
entry point, its parameter structs have the layout the ctypes binding assumes, and argument
errors come back as status codes before any CUDA work is enqueued."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from mamba_cpu_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mamba_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"MB200_API\s+[\w\s\*]+?\b(mb200_\w+)\s*\(", src)))


def test_every_declared_symbol_is_exported_and_bound():
    names = _declared()
    assert len(names) >= 13, names
    for n in names:
        assert hasattr(_lib.lib, n), f"{n} not exported by {_lib.LIB_PATH}"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature in mamba_cpu_b200._lib"
    assert set(_lib.SIGNATURES) == set(names)


def test_exported_symbols_are_only_the_abi():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l and l.split()[-1].startswith("mb200_")}
    assert exported == set(_declared())


_STRUCTS = {
    "mb200_scan_fwd_params": _lib.ScanFwdParams,
    "mb200_scan_bwd_params": _lib.ScanBwdParams,
    "mb200_conv1d_params": _lib.Conv1dParams,
    "mb200_state_update_params": _lib.StateUpdateParams,
    "mb200_conv1d_update_params": _lib.Conv1dUpdateParams,
    "mb200_ssd_params": _lib.SsdParams,
}


def test_struct_layout_matches_header():
    """Compile a probe against the header with the host C compiler and compare sizeof/offsetof."""
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mamba_b200.h"', "int main(void) {"]
    for cname, py in _STRUCTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as td:
        src = os.path.join(td, "probe.c")
        exe = os.path.join(td, "probe")
        open(src, "w").write("\n".join(lines))
        cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
        subprocess.run([cc, "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        got = dict(l.split() for l in subprocess.run([exe], capture_output=True, text=True, check=True)
                   .stdout.splitlines())
    for cname, py in _STRUCTS.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def _fwd(**kw):
    p = _lib.ScanFwdParams()
    p.u = p.delta = p.A = p.B = p.C = p.out = 0x1000
    p.batch, p.dim, p.seqlen, p.dstate, p.ngroups = 1, 4, 8, 4, 1
    p.B_batch_stride = p.C_batch_stride = 32
    p.B_group_stride = p.C_group_stride = 32
    p.B_dstate_stride = p.C_dstate_stride = 8
    p.B_seqlen_stride = p.C_seqlen_stride = 1
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,status", [
    (dict(dstate=17), 5),
    (dict(dstate=0), 2),
    (dict(ngroups=3), 2),
    (dict(batch=-1), 2),
    (dict(io_dtype=7), 3),
    (dict(io_dtype=_lib.BF16, bc_dtype=_lib.F16), 3),
    (dict(u=None), 1),
    (dict(out=None), 1),
])
def test_scan_fwd_rejects_bad_arguments_before_launch(kw, status):
    # Validation runs before any CUDA call, so this is safe without a GPU.
    assert _lib.lib.mb200_selective_scan_fwd(_fwd(**kw), None) == status
    assert _lib.status_string(status)


def test_scan_bwd_workspace_and_validation():
    b = _lib.ScanBwdParams()
    b.fwd = _fwd()
    assert _lib.lib.mb200_selective_scan_bwd_workspace_size(b) == 0  # dout etc. missing
    b.dout = b.du = b.ddelta = b.dA = b.dB = b.dC = 0x2000
    need = _lib.lib.mb200_selective_scan_bwd_workspace_size(b)
    assert need > 0 and need % 256 == 0
    assert _lib.lib.mb200_selective_scan_bwd(b, None, 0, None) == 6
    assert _lib.lib.mb200_selective_scan_bwd(b, 0x10001, need, None) == 6  # misaligned
    b.fwd.z = 0x3000  # z given but dz missing
    assert _lib.lib.mb200_selective_scan_bwd(b, 0x10000, need, None) == 1


def test_conv_and_decode_validation():
    c = _lib.Conv1dParams()
    c.x = c.weight = c.out = 0x1000
    c.batch, c.dim, c.seqlen, c.width = 1, 4, 8, 9
    assert _lib.lib.mb200_causal_conv1d_fwd(c, None) == 5
    c.width = 0
    assert _lib.lib.mb200_causal_conv1d_fwd(c, None) == 2
    u = _lib.Conv1dUpdateParams()
    u.x = u.conv_state = u.weight = u.out = 0x1000
    u.batch, u.dim, u.seqlen, u.state_len, u.width = 1, 4, 1, 2, 4
    assert _lib.lib.mb200_causal_conv1d_update(u, None) == 2  # state_len < width - 1
    s = _lib.StateUpdateParams()
    s.state = s.x = s.dt = s.A = s.B = s.C = s.out = 0x1000
    s.batch, s.dim, s.dstate, s.ngroups = 1, 4, _lib.DECODE_MAX_DSTATE + 1, 1  # beyond the decode limit
    assert _lib.lib.mb200_selective_state_update(s, None) == 5


def test_version_and_status_strings():
    assert _lib.lib.mb200_version() >> 16 == 1
    for st in range(8):
        assert _lib.status_string(st)
    assert _lib.status_string(99) == "unknown status"
