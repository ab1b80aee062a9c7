"""Parity at the benchmark's full sizes (BASELINE configs 3 and 4), where the CPU oracle is too slow
for whole tensors: one full head is checked against the same fp32 formulas evaluated on the GPU
(the oracle's torch code on CUDA tensors, or a dense fp32 attention), and every head is checked
through size-independent properties (entropy in [0, ln N], outputs inside the convex hull of V)."""
import math

import pytest
import torch

import oracle
from conftest import max_rel_err
from vmonarch_b200 import flash_entropy_attention, vmonarch_attention
from vmonarch_b200.configs import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu


def test_fea_config3_full_size():
    w = WORKLOADS["fea32k"]  # B=1, H=24, N=32768, D=128
    dev = torch.device("cuda")
    q, k, v, do, de = (t.to(dev) for t in make_inputs(w, seed=0))
    leaves = [t.requires_grad_() for t in (q, k, v)]
    o, e = flash_entropy_attention(*leaves)
    dq, dk, dv = torch.autograd.grad((o, e), leaves, (do, de))
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(e).all()
    assert (e >= -1e-3).all() and (e <= math.log(w.N) + 1e-3).all()
    vmax, vmin = v.detach().float().amax(-2, keepdim=True), v.detach().float().amin(-2, keepdim=True)
    assert (o.float() <= vmax + 1e-2).all() and (o.float() >= vmin - 1e-2).all()
    # head 0 in full against dense fp32 attention (same formulas as the oracle) on the GPU
    h = 0
    qh, kh, vh = (t.detach()[0, h].float().requires_grad_() for t in (q, k, v))
    o_r, e_r = oracle.entropy_attention(qh, kh, vh, w.D ** -0.5)
    g_r = torch.autograd.grad((o_r * do[0, h].float()).sum() + (e_r * de[0, h]).sum(), (qh, kh, vh))
    assert (o[0, h].float() - o_r).abs().max() <= 2e-2 and (o[0, h].float() - o_r).abs().mean() <= 2e-3
    assert (e[0, h] - e_r).abs().max() <= 1e-3 * e_r.abs().max()
    for g, gr in zip((dq, dk, dv), g_r):
        assert max_rel_err(g[0, h], gr) <= 3e-2
        assert (g[0, h].float() - gr).abs().max() <= max(5e-2, 8e-3 * gr.abs().max().item())


def test_vmonarch_config4_one_full_head():
    w = WORKLOADS["dit14b"]  # m=21, b=1560, D=128, 2 iterations, r=1560
    dev = torch.device("cuda")
    q, k, v, do, _ = (t.to(dev) for t in make_inputs(w, seed=1, heads=range(3, 4)))
    leaves = [t.requires_grad_() for t in (q, k, v)]
    z = vmonarch_attention(*leaves, w.m, w.b, w.iters, recompute_tokens=w.recompute)
    grads = torch.autograd.grad(z, leaves, do)
    ref_leaves = [t.detach().float().requires_grad_() for t in (q, k, v)]
    z_r = oracle.vmonarch_attention(*ref_leaves, w.m, w.b, w.iters, recompute_tokens=w.recompute)
    g_r = torch.autograd.grad(z_r, ref_leaves, do.float())
    assert max_rel_err(z, z_r) <= 3e-2
    for g, gr in zip(grads, g_r):
        assert max_rel_err(g, gr) <= 5e-2


def test_vmonarch_config5_forward_one_head():
    w = WORKLOADS["long720p"]  # m=32, b=3600, 3 iterations, r=3600
    dev = torch.device("cuda")
    q, k, v, _, _ = (t.to(dev) for t in make_inputs(w, seed=2, heads=range(0, 1)))
    with torch.no_grad():
        z = vmonarch_attention(q, k, v, w.m, w.b, w.iters, recompute_tokens=w.recompute)
        z_r = oracle.vmonarch_attention(q.float(), k.float(), v.float(), w.m, w.b, w.iters,
                                        recompute_tokens=w.recompute)
    assert max_rel_err(z, z_r) <= 3e-2
