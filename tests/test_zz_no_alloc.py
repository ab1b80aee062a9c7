"""vmb_fea_bwd_noalloc: the FlashEntropyAttention backward for callers that cannot allocate.

Hosts such as engine plugins (whose enqueue hook may not allocate because the framework owns all
device memory) or foreign-language bindings (which can only pass the user's tensors) cannot give
vmb_fea_bwd its scratch workspace; this entry point uses a fixed buffer inside the library instead.
The test calls it through the C ABI twice in a row (the second call sees the first call's leftover
scratch) and checks each result against vmb_fea_bwd with an ordinary caller-provided workspace,
within the tolerances of the FlashEntropyAttention parity tests. It lives in its own file named to
be collected last and needs nothing from the other tests.
"""
import ctypes

import pytest
import torch

from vmonarch_b200 import _native as N
from vmonarch_b200 import ops

pytestmark = pytest.mark.gpu


def _bwd_args(q, k, v, o, do, lse, ent, de, dq, dk, dv, sm_scale):
    a = N.FeaBwdArgs()
    B, H, S, D = q.shape
    Dv = v.shape[-1]
    a.q, a.q_bs = q.data_ptr(), S * D
    a.k, a.k_bs = k.data_ptr(), S * D
    a.v, a.v_bs = v.data_ptr(), S * Dv
    a.o, a.o_bs = o.data_ptr(), S * Dv
    a.dout, a.do_bs = do.data_ptr(), S * Dv
    a.lse, a.ent, a.dent = lse.data_ptr(), ent.data_ptr(), de.data_ptr()
    a.grad_q, a.grad_q_bs = dq.data_ptr(), S * D
    a.grad_k, a.grad_k_bs = dk.data_ptr(), S * D
    a.grad_v, a.grad_v_bs = dv.data_ptr(), S * Dv
    a.batch, a.n_q, a.n_kv = B * H, S, S
    a.d, a.dv, a.dv1, a.dtype = D, Dv, Dv, N.VMB_DTYPE_BF16
    a.grad_mode, a.v_is_k = 0, 0
    a.sm_scale = sm_scale
    return a


def _close(x, ref):
    err = (x.float() - ref.float()).abs().max().item()
    scale = max(ref.float().abs().max().item(), 1e-3)
    return err <= 3e-2 * scale and err <= max(5e-2, 8e-3 * scale)


def test_noalloc_backward_matches_workspace_backward():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator().manual_seed(11)
    B, H, S, D = 2, 3, 333, 128
    q, k, v = (torch.randn(B, H, S, D, generator=gen).bfloat16().to(dev) for _ in range(3))
    do = torch.randn(B, H, S, D, generator=gen).bfloat16().to(dev)
    de = torch.randn(B, H, S, generator=gen).to(dev)
    sm_scale = D ** -0.5
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, device=dev)
    ent = torch.empty(B, H, S, device=dev)
    ops.fea_fwd(q, k, v, o, lse, ent, sm_scale)
    stream = N.stream_ptr(dev)

    # existing entry point, workspace allocated by the caller
    ref = [torch.empty_like(t) for t in (q, k, v)]
    a = _bwd_args(q, k, v, o, do, lse, ent, de, *ref, sm_scale)
    nbytes = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    N.check(N.lib.vmb_fea_bwd(ctypes.byref(a), stream), "vmb_fea_bwd")

    for _ in range(2):  # two calls in a row share (and inherit) the built-in scratch
        got = [torch.full_like(t, float("nan")) for t in (q, k, v)]
        b = _bwd_args(q, k, v, o, do, lse, ent, de, *got, sm_scale)
        N.check(N.lib.vmb_fea_bwd_noalloc(ctypes.byref(b), stream), "vmb_fea_bwd_noalloc")
        torch.cuda.synchronize(dev)
        for g, r in zip(got, ref):
            assert torch.isfinite(g.float()).all()
            assert _close(g, r)


def test_noalloc_rejects_requests_beyond_its_scratch():
    # Placeholder pointers that are NOT 16-byte aligned: should the size check ever let this request
    # through, vmb_fea_bwd's own validation rejects it before anything is launched on the device.
    a = N.FeaBwdArgs()
    a.q = a.k = a.v = a.o = a.dout = a.lse = a.grad_q = a.grad_k = a.grad_v = 8
    # 64 sequences of 2^20 queries: at least 768 MiB of scratch on every backward path
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = 64, 1 << 20, 1 << 20, 128, 128, 128
    a.grad_mode, a.sm_scale = 0, 0.1
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) > 32 << 20
    assert N.lib.vmb_fea_bwd_noalloc(ctypes.byref(a), None) == 1
    assert b"scratch" in N.lib.vmb_last_error()
