"""Backward calls split over their batch under the workspace bound give the same gradients as one call.

Every sequence of a call is an independent problem and the split keeps the kernel route (dS^T
stored by the dK/dV kernel, dQ formed from it by a GEMM), so with deterministic kernels the
gradients are bitwise equal."""
import ctypes

import pytest
import torch

from vmonarch_b200 import _native as N
from vmonarch_b200 import flash_entropy_attention, ops, vmonarch_attention

pytestmark = pytest.mark.gpu


def _with_limit(nbytes, fn):
    old = ops.workspace_limit()
    ops.set_workspace_limit(nbytes)
    try:
        return fn()
    finally:
        ops.set_workspace_limit(old)


def test_chunked_fea_backward_matches_one_call():
    # 80 sequences of 1024 with separate V: 640 query tiles, dS^T 168 MB; a 100 MB bound splits the
    # call in two halves that each keep the dS^T route
    H, S, D = 80, 1024, 128
    a = N.FeaBwdArgs()
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = H, S, S, D, D, D
    assert _with_limit(100 << 20, lambda: ops.bwd_plan(a))[0] == H // 2
    gen = torch.Generator(device="cuda").manual_seed(3)
    q, k, v, do = (torch.randn(1, H, S, D, device="cuda", generator=gen).bfloat16() for _ in range(4))
    de = torch.randn(1, H, S, device="cuda", generator=gen)

    def grads():
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        o, e = flash_entropy_attention(*leaves)
        return torch.autograd.grad((o, e), leaves, (do, de))

    one = grads()
    split = _with_limit(100 << 20, grads)
    torch.cuda.synchronize()
    for g, r in zip(split, one):
        assert torch.equal(g, r)


def test_chunked_vmonarch_backward_matches_one_call():
    # the last R step (values [k | v], 64 grid rows of 1000 tokens: dS^T 134 MB) and the recompute
    # split under a 40 MB bound; deterministic mode keeps every other kernel bitwise reproducible
    m, b, H = 8, 1000, 8
    gen = torch.Generator(device="cuda").manual_seed(4)
    q, k, v, dz = (torch.randn(1, H, m * b, 128, device="cuda", generator=gen).bfloat16() for _ in range(4))

    def grads():
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        z = vmonarch_attention(*leaves, m, b, 2, recompute_tokens=b)
        return (z, *torch.autograd.grad(z, leaves, dz))

    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        one = grads()
        split = _with_limit(40 << 20, grads)
        torch.cuda.synchronize()
    finally:
        torch.use_deterministic_algorithms(False)
    for g, r in zip(split, one):
        assert torch.equal(g, r)
