"""The C-ABI library: loads without a GPU, exports every declared symbol, struct layouts agree with
the ctypes mirror, and argument validation rejects bad calls before any CUDA work is issued."""
import ctypes
import re
import subprocess
import tempfile
from pathlib import Path

import pytest

from vmonarch_b200 import _native as N

HEADER = Path(__file__).resolve().parent.parent / "include" / "vmonarch_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(vmb_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_reports_abi():
    assert N.LIB_PATH.exists()
    assert N.lib.vmb_abi_version() == N.ABI_VERSION == 7


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 8
    for name in names:
        assert hasattr(N.lib, name), f"{name} not exported"
        assert name in N.SIGNATURES, f"{name} has no ctypes binding"
    assert set(N.SIGNATURES) == set(names)


STRUCTS = {"vmb_fea_fwd_args": N.FeaFwdArgs, "vmb_fea_bwd_args": N.FeaBwdArgs, "vmb_lstep_args": N.LstepArgs,
           "vmb_view": N.View, "vmb_fea_layout": N.FeaLayout, "vmb_lstep_layout": N.LstepLayout}


def test_struct_layouts_match_c_header():
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for cname, pytype in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in pytype._fields_:
            lines.append(f'printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as tmp:
        src, exe = Path(tmp) / "layout.c", Path(tmp) / "layout"
        src.write_text("\n".join(lines))
        subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", str(src), "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    got = {}
    for line in out.splitlines():
        cname, field, val = line.split()
        got[(cname, field)] = int(val)
    for cname, pytype in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(pytype), cname
        for field, _ in pytype._fields_:
            assert got[(cname, field)] == getattr(pytype, field).offset, (cname, field)


def fwd_args(**over):
    a = N.FeaFwdArgs()
    a.q = a.k = a.v = a.o = 256
    a.batch, a.n_q, a.n_kv = 1, 128, 128
    a.d, a.dv, a.dv1, a.dtype = 64, 64, 64, N.VMB_DTYPE_BF16
    a.sm_scale = 0.125
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over, code", [
    (dict(dtype=7), 1),
    (dict(d=96), 2),
    (dict(d=128, dv=64), 2),
    (dict(n_kv=0), 1),
    (dict(dv1=32), 1),
    (dict(q=None), 1),
    (dict(q=258), 1),
    (dict(q_bs=3), 1),
])
def test_fea_fwd_rejects_bad_arguments_without_touching_cuda(over, code):
    rc = N.lib.vmb_fea_fwd(ctypes.byref(fwd_args(**over)), None)
    assert rc == code
    assert N.lib.vmb_last_error()


def test_fea_fwd_empty_batch_is_a_no_op():
    assert N.lib.vmb_fea_fwd(ctypes.byref(fwd_args(batch=0)), None) == 0
    assert N.lib.vmb_fea_fwd(ctypes.byref(fwd_args(n_q=0)), None) == 0
    assert N.lib.vmb_fea_fwd(None, None) == 1


def test_fea_bwd_workspace_and_validation():
    a = N.FeaBwdArgs()
    # D = 32 runs on the warp-level MMA kernels: c and g per row, and an fp32 dQ in grad_mode 0
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = 3, 100, 100, 32, 32, 32
    a.grad_mode = 0
    rows = 300
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == 2 * 1280 + ((rows * 32 * 4 + 255) // 256) * 256
    a.grad_mode = 1
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == 2 * 1280
    # D = Dv = 64 runs the tcgen05 kernels over 64-column maps: the folded statistics planes only
    a.d, a.dv, a.dv1, a.grad_mode = 64, 64, 64, 0
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == 3 * ((3 * 128 * 4 + 255) // 256) * 256
    # D = 64 with Dv = 128 (separate values) takes the same kernels
    a.dv = a.dv1 = 128
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == 3 * ((3 * 128 * 4 + 255) // 256) * 256
    # ... and so does D = 64 with V aliasing K and a second value tensor ([K | V2] tiles), except in
    # the finalize mode, which the warp-level kernels serve (c and g per row)
    a.dv, a.dv1, a.v_is_k, a.grad_mode = 128, 64, 1, 2
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == 3 * ((3 * 128 * 4 + 255) // 256) * 256
    a.grad_mode = 3
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == 2 * 1280
    a.dv = a.dv1 = 64
    a.v_is_k, a.grad_mode = 0, 0
    # D = 128 runs on the tcgen05 kernels: three folded statistics planes of 3 x round_up(100, 128)
    # rows. Three query tiles cannot fill the GPU, so the dS^T route is not taken: no dS^T buffer.
    a.d, a.dv, a.dv1 = 128, 128, 128
    planes = 3 * ((3 * 128 * 4 + 255) // 256) * 256
    assert N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a)) == planes
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == planes
    # 400 sequences (400 query tiles, two or more per SM): the preferred size adds the dS^T buffer
    # (2 bytes x round_up(100, 128) keys x round_up(100, 64) queries per sequence, on a 256-byte
    # boundary); the minimum does not
    a.batch = 400
    planes = 3 * ((400 * 128 * 4 + 255) // 256) * 256
    assert N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a)) == planes
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) == planes + 400 * 128 * 128 * 2 + 256
    a.batch = 3
    a.d, a.dv, a.dv1 = 64, 64, 64
    a.q = a.k = a.v = a.o = a.dout = a.lse = a.grad_q = a.grad_k = a.grad_v = 256
    a.dtype = 0
    a.v_is_k = 1                      # v_is_k with a separate grad_v is rejected
    assert N.lib.vmb_fea_bwd(ctypes.byref(a), None) == 1
    a.v_is_k = 0
    a.grad_mode = 4                   # modes are 0 (16-bit), 1 (fp32 add), 2 (fp32 overwrite), 3 (finalize)
    assert N.lib.vmb_fea_bwd(ctypes.byref(a), None) == 1
    assert b"grad_mode" in N.lib.vmb_last_error()
    a.grad_mode = 3                   # finalize without its fp32 accumulators
    assert N.lib.vmb_fea_bwd(ctypes.byref(a), None) == 1
    assert b"accumulator" in N.lib.vmb_last_error()
    a.grad_mode = 1
    a.workspace, a.workspace_bytes = 256, 16   # too small
    assert N.lib.vmb_fea_bwd(ctypes.byref(a), None) == 1
    assert b"workspace" in N.lib.vmb_last_error()


def test_lstep_validation():
    a = N.LstepArgs()
    a.q = a.out = a.ent = a.u = 256
    a.bh, a.m, a.b, a.d, a.dw, a.dtype = 1, 129, 4, 64, 64, 0
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 2     # m > 128
    a.m, a.d, a.dw = 65, 32, 32
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 2     # m > 64 on the generic kernel (d = 32)
    assert b"> 64" in N.lib.vmb_last_error()
    a.m = 4
    a.d = a.dw = 256
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 2     # d = 256 (D + Dv <= 256 in VMonarch)
    a.d = a.dw = 48
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 2     # d = 48
    a.d, a.dw, a.last = 64, 100, 1
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 2     # value width 36
    a.dw, a.last = 64, 0
    a.bh = 0
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 0     # nothing to do
    a.bh, a.u = 1, None
    assert N.lib.vmb_lstep_fwd(ctypes.byref(a), None) == 1
    assert N.lib.vmb_lstep_bwd(ctypes.byref(a), None) == 1     # no gradients given
    assert N.lib.vmb_cast_f32(None, 0, None, 0, 1, 6, 0, None) == 1


def test_fea_fwd_workspace_query():
    # The workspace only exists for the d = dv = 128 kernel when a key-range split pays off: few
    # query tiles over many keys. Many query tiles, other head dims and empty calls need none.
    a = N.FeaFwdArgs()
    a.q, a.k, a.v = 256, 512, 768
    a.q_bs = a.k_bs = a.v_bs = 0
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = 2, 128, 32768, 128, 128, 128
    assert N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a)) > 0
    a.batch, a.n_q, a.n_kv = 840, 1560, 1560
    assert N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a)) == 0
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = 2, 128, 32768, 64, 64, 64
    assert N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a)) == 0
    a.n_q = 0
    assert N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a)) == 0
    assert N.lib.vmb_fea_fwd_workspace_bytes(None) == -1
