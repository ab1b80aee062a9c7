"""vmb_fea_bwd_noalloc: the FlashEntropyAttention backward for callers that cannot allocate.

Hosts such as engine plugins (whose enqueue hook may not allocate because the framework owns all
device memory) or foreign-language bindings (which can only pass the user's tensors) cannot give
vmb_fea_bwd its scratch workspace; this entry point uses a fixed buffer inside the library instead.
The test calls it through the C ABI on calls of different shapes in a row, so each call finds the
previous one's leftover scratch, on three kernel routes: the tcgen05 backward (d = 128), the
mma.sync backward at d = 32 (whose fp32 dQ accumulator in the scratch must be cleared on every
call) and the last VMonarch R step (V aliasing K with a second value tensor, dv = 256), whose dS^T
buffer fits the built-in scratch at this size. Each result is checked against vmb_fea_bwd with an
ordinary caller-provided workspace of the same route, within the tolerances of the
FlashEntropyAttention parity tests. The file is named to be collected last and needs nothing from
the other tests.
"""
import ctypes

import pytest
import torch

from vmonarch_b200 import _native as N
from vmonarch_b200 import ops

pytestmark = pytest.mark.gpu

SCRATCH = 32 << 20


class Case:
    """Inputs, forward outputs and backward arguments of one FlashEntropyAttention call."""

    def __init__(self, seed, batch, n, d, dv, v_is_k=False):
        dev = torch.device("cuda", 0)
        gen = torch.Generator().manual_seed(seed)
        rnd = lambda *s: torch.randn(*s, generator=gen).to(dev)  # noqa: E731
        self.batch, self.n, self.d, self.dv, self.v_is_k = batch, n, d, dv, v_is_k
        self.q, self.k = rnd(batch, n, d).bfloat16(), rnd(batch, n, d).bfloat16()
        # with V aliasing K the values are [k | v2]; otherwise v is its own tensor
        self.v = self.k if v_is_k else rnd(batch, n, dv).bfloat16()
        self.v2 = rnd(batch, n, dv - d).bfloat16() if v_is_k else None
        self.do, self.de = rnd(batch, n, dv).bfloat16(), rnd(batch, n)
        self.scale = d ** -0.5
        self.o = torch.empty(batch, n, dv, device=dev, dtype=torch.bfloat16)
        self.lse, self.ent = torch.empty(batch, n, device=dev), torch.empty(batch, n, device=dev)
        ops.fea_fwd(self.q, self.k, self.v, self.o, self.lse, self.ent, self.scale, v2=self.v2)

    def grads_like(self, fill):
        shapes = [self.q, self.k] + ([self.v2] if self.v_is_k else [self.v])
        return [torch.full_like(t, fill) for t in shapes]

    def args(self, grads):
        dq, dk, dvx = grads
        a = N.FeaBwdArgs()
        n, d, dv = self.n, self.d, self.dv
        a.q, a.q_bs = self.q.data_ptr(), n * d
        a.k, a.k_bs = self.k.data_ptr(), n * d
        a.o, a.o_bs = self.o.data_ptr(), n * dv
        a.dout, a.do_bs = self.do.data_ptr(), n * dv
        a.lse, a.ent, a.dent = self.lse.data_ptr(), self.ent.data_ptr(), self.de.data_ptr()
        a.grad_q, a.grad_q_bs = dq.data_ptr(), n * d
        a.grad_k, a.grad_k_bs = dk.data_ptr(), n * d
        if self.v_is_k:
            a.v, a.v_bs, a.dv1, a.v_is_k = self.k.data_ptr(), n * d, d, 1
            a.v2, a.v2_bs = self.v2.data_ptr(), n * (dv - d)
            a.grad_v2, a.grad_v2_bs = dvx.data_ptr(), n * (dv - d)
        else:
            a.v, a.v_bs, a.dv1 = self.v.data_ptr(), n * dv, dv
            a.grad_v, a.grad_v_bs = dvx.data_ptr(), n * dv
        a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dtype = self.batch, n, n, d, dv, N.VMB_DTYPE_BF16
        a.grad_mode, a.sm_scale, a.deterministic = 0, self.scale, 1
        return a

    def with_workspace(self, preferred):
        """Gradients from vmb_fea_bwd with a caller-provided workspace (preferred or minimal size)."""
        grads = self.grads_like(0.0)
        a = self.args(grads)
        query = N.lib.vmb_fea_bwd_workspace_bytes if preferred else N.lib.vmb_fea_bwd_min_workspace_bytes
        nbytes = query(ctypes.byref(a))
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=self.q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
        N.check(N.lib.vmb_fea_bwd(ctypes.byref(a), N.stream_ptr(self.q.device)), "vmb_fea_bwd")
        torch.cuda.synchronize()
        return grads

    def no_alloc(self):
        grads = self.grads_like(float("nan"))
        a = self.args(grads)
        N.check(N.lib.vmb_fea_bwd_noalloc(ctypes.byref(a), N.stream_ptr(self.q.device)), "vmb_fea_bwd_noalloc")
        torch.cuda.synchronize()
        return grads


def _close(x, ref):
    err = (x.float() - ref.float()).abs().max().item()
    scale = max(ref.float().abs().max().item(), 1e-3)
    return err <= 3e-2 * scale and err <= max(5e-2, 8e-3 * scale)


def test_noalloc_backward_matches_workspace_backward():
    torch.cuda.set_device(0)
    cases = [Case(11, 6, 333, 128, 128),               # tcgen05 backward, separate V
             Case(12, 4, 200, 32, 32),                 # mma.sync backward: dQ accumulator in the scratch
             Case(13, 8, 1000, 128, 256, v_is_k=True)]  # last R step: dS^T in the scratch
    dst = cases[2]
    a = dst.args(dst.grads_like(0.0))
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) <= SCRATCH
    assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a)) > N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a))
    refs = [c.with_workspace(preferred=True) for c in cases]
    # each call follows a call of another shape, whose scratch contents it inherits; every case runs
    # twice, and case 0 twice in a row at the end
    for i in (0, 1, 2, 1, 2, 0, 0):
        got = cases[i].no_alloc()
        for g, r in zip(got, refs[i]):
            assert torch.isfinite(g.float()).all(), i
            assert _close(g, r), i


def test_noalloc_rejects_requests_beyond_its_scratch():
    # Placeholder pointers that are NOT 16-byte aligned: should the size check ever let this request
    # through, vmb_fea_bwd's own validation rejects it before anything is launched on the device.
    a = N.FeaBwdArgs()
    a.q = a.k = a.v = a.o = a.dout = a.lse = a.grad_q = a.grad_k = a.grad_v = 8
    # 64 sequences of 2^20 queries: at least 768 MiB of scratch on every backward path
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = 64, 1 << 20, 1 << 20, 128, 128, 128
    a.grad_mode, a.sm_scale = 0, 0.1
    assert N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a)) > SCRATCH
    assert N.lib.vmb_fea_bwd_noalloc(ctypes.byref(a), None) == 1
    assert b"scratch" in N.lib.vmb_last_error()
