"""The CPU oracle against the golden vectors produced by the reference itself (no GPU)."""
import pytest
import torch
import torch.nn.functional as F

import oracle
from conftest import FEA_GOLDEN, VM_GOLDEN, load_golden


@pytest.mark.parametrize("name", FEA_GOLDEN)
def test_oracle_fea_matches_reference_golden(name):
    g = load_golden(name)
    D = g["q"].shape[-1]
    leaves = [g[t].clone().requires_grad_() for t in ("q", "k", "v")]
    o, e = oracle.entropy_attention(*leaves, D ** -0.5)
    grads = torch.autograd.grad((o * g["do"]).sum() + (e * g["de"]).sum(), leaves)
    for got, key in zip((o, e, *grads), ("o", "e", "dq", "dk", "dv")):
        torch.testing.assert_close(got.detach(), g[key], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", VM_GOLDEN)
def test_oracle_vmonarch_matches_reference_golden(name):
    g = load_golden(name)
    B, H, m, b, D, iters, r, _ = g["meta"].tolist()
    leaves = [g[t].clone().requires_grad_() for t in ("q", "k", "v")]
    z = oracle.vmonarch_attention(*leaves, m, b, iters, recompute_tokens=r)
    grads = torch.autograd.grad((z * g["dz"]).sum(), leaves)
    for got, key in zip((z, *grads), ("z", "dq", "dk", "dv")):
        ref = g[key]
        assert (got.detach() - ref).abs().max() <= 1e-4 * max(1.0, ref.abs().max().item())


def test_oracle_entropy_attention_is_naive_softmax_attention():
    # config 1 of the benchmark: B=1, H=2, N=256, D=64, seed 0 (CPU fp32 plumbing run)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 2, 256, 64, generator=g) for _ in range(3))
    o, e = oracle.entropy_attention(q, k, v, 64 ** -0.5)
    p = torch.softmax(q @ k.transpose(-1, -2) / 8.0, -1)
    torch.testing.assert_close(o, p @ v, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(e, -(p * p.log()).sum(-1), rtol=1e-5, atol=1e-5)
    assert e.shape == (1, 2, 256)
    z = oracle.vmonarch_attention(q, k, v, 4, 64, 2, recompute_tokens=64)
    assert z.shape == (1, 2, 256, 64)


def test_oracle_recompute_rows_are_exact_attention():
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, 1, 96, 64, generator=g) for _ in range(3))
    z = oracle.vmonarch_attention(q, k, v, 3, 32, 2, recompute_tokens=40)
    exact = F.scaled_dot_product_attention(q, k, v)
    torch.testing.assert_close(z[:, :, :40], exact[:, :, :40])
    z_all = oracle.vmonarch_attention(q, k, v, 3, 32, 2, recompute_tokens=1000)
    torch.testing.assert_close(z_all, exact)


def test_oracle_edge_errors():
    q = torch.randn(1, 1, 64, 64)
    with pytest.raises(AssertionError):
        oracle.vmonarch_attention(q, q, q, 3, 32)
    with pytest.raises(UnboundLocalError):
        oracle.vmonarch_attention(q, q, q, 2, 32, num_iters=0)


def test_oracle_entropy_bounds_and_rows():
    g = torch.Generator().manual_seed(2)
    q, k, v = (torch.randn(1, 1, 300, 64, generator=g) * 3 for _ in range(3))
    o, e = oracle.entropy_attention(q, k, v, 0.125)
    assert (e >= -1e-5).all() and (e <= torch.log(torch.tensor(300.0)) + 1e-5).all()
    rows = torch.tensor([0, 7, 299])
    o2, e2 = oracle.entropy_attention_rows(q, k, v, 0.125, rows)
    torch.testing.assert_close(o2, o[..., rows, :])
    torch.testing.assert_close(e2, e[..., rows])
