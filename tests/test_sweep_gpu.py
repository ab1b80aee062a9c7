"""Seeded random sweep of FlashEntropyAttention and VMonarch shapes against the fp32 oracle.

The fixed-shape tests pin each kernel route at chosen sizes; this sweep draws the options together
(batch, heads, ragged lengths, head dims, fp16 / bf16, token-major views, values aliasing keys, a
custom scale; Monarch grids, iteration counts and recompute lengths) so that combinations no
fixed test names are also held to the same tolerances (test_fea_gpu.check, test_vmonarch_gpu.check).
Each case prints its draw in the test id, so a failure reproduces from its seed alone.
"""
import random

import pytest
import torch

import oracle
from test_fea_gpu import check as check_fea
from test_vmonarch_gpu import check as check_vm
from vmonarch_b200 import flash_entropy_attention, vmonarch_attention

pytestmark = pytest.mark.gpu

FEA_LENGTHS = [1, 2, 31, 64, 65, 127, 129, 200, 255, 257, 500, 777, 1024, 1560, 2049, 3000]
FEA_DIMS = [(64, 64), (128, 128), (128, 256), (64, 128), (32, 32), (16, 64)]


def fea_draw(seed):
    r = random.Random(seed)
    D, Dv = r.choice(FEA_DIMS)
    return dict(B=r.choice([1, 2]), H=r.choice([1, 2, 3]), N=r.choice(FEA_LENGTHS), D=D, Dv=Dv,
                dtype=r.choice(["bf16", "fp16"]), token_major=r.random() < 0.4,
                alias=D == Dv and r.random() < 0.3, scale=r.choice([None, None, 0.05, 0.2]))


def as_layout(x, token_major):
    """x, or x stored as (B, N, H, C) and seen through transpose(1, 2)."""
    return x.transpose(1, 2).contiguous().transpose(1, 2) if token_major else x


FEA_CASES = [fea_draw(s) for s in range(48)]


@pytest.mark.parametrize("case", FEA_CASES, ids=[f"s{i}-" + "-".join(f"{k}{v}" for k, v in c.items())
                                                 for i, c in enumerate(FEA_CASES)])
def test_fea_sweep(case):
    c = case
    gen = torch.Generator().manual_seed(1000 + c["N"] + 7 * c["D"])
    B, H, N, D, Dv = c["B"], c["H"], c["N"], c["D"], c["Dv"]
    dtype = torch.bfloat16 if c["dtype"] == "bf16" else torch.float16
    q, k = (torch.randn(B, H, N, D, generator=gen).to(dtype).float() for _ in range(2))
    v = k if c["alias"] else torch.randn(B, H, N, Dv, generator=gen).to(dtype).float()
    do, de = torch.randn(B, H, N, Dv, generator=gen), torch.randn(B, H, N, generator=gen)
    scale = c["scale"] if c["scale"] is not None else D ** -0.5

    qd, kd = (as_layout(t.cuda().to(dtype), c["token_major"]).requires_grad_() for t in (q, k))
    if c["alias"]:
        o, e = flash_entropy_attention(qd, kd, kd, sm_scale=c["scale"])
        leaves = [qd, kd]
    else:
        vd = as_layout(v.cuda().to(dtype), c["token_major"]).requires_grad_()
        o, e = flash_entropy_attention(qd, kd, vd, sm_scale=c["scale"])
        leaves = [qd, kd, vd]
    grads = torch.autograd.grad((o.float() * do.cuda()).sum() + (e * de.cuda()).sum(), leaves)
    torch.cuda.synchronize()
    got = [t.detach().float().cpu() for t in (o, e, *grads)]

    ref_leaves = [t.clone().requires_grad_() for t in ((q, k) if c["alias"] else (q, k, v))]
    o_r, e_r = oracle.entropy_attention(ref_leaves[0], ref_leaves[1], ref_leaves[-1], scale)
    g_r = torch.autograd.grad((o_r * do).sum() + (e_r * de).sum(), ref_leaves)
    check_fea(got, [o_r.detach(), e_r.detach(), *(g.detach() for g in g_r)])


def vm_draw(seed):
    r = random.Random(10_000 + seed)
    m = r.randint(2, 128)
    b = r.choice([16, 33, 64, 100, 128, 129, 200, 257])
    N = m * b
    return dict(B=r.choice([1, 2]), H=r.choice([1, 2]), m=m, b=b, iters=r.choice([1, 2, 3]),
                r=r.choice([0, b, min(N, 2 * b + 5), r.randint(1, N)]), D=r.choice([64, 128, 128]),
                dtype=r.choice(["bf16", "bf16", "fp16"]), token_major=r.random() < 0.3)


VM_CASES = [vm_draw(s) for s in range(24)]


@pytest.mark.parametrize("case", VM_CASES, ids=[f"s{i}-" + "-".join(f"{k}{v}" for k, v in c.items())
                                                for i, c in enumerate(VM_CASES)])
def test_vmonarch_sweep(case):
    c = case
    B, H, m, b, D = c["B"], c["H"], c["m"], c["b"], c["D"]
    N = m * b
    dtype = torch.bfloat16 if c["dtype"] == "bf16" else torch.float16
    gen = torch.Generator().manual_seed(2000 + N + D)
    q, k, v = (torch.randn(B, H, N, D, generator=gen).to(dtype).float() for _ in range(3))
    dz = torch.randn(B, H, N, D, generator=gen)

    leaves = [as_layout(t.cuda().to(dtype), c["token_major"]).requires_grad_() for t in (q, k, v)]
    z = vmonarch_attention(*leaves, m, b, c["iters"], recompute_tokens=c["r"])
    grads = torch.autograd.grad((z.float() * dz.cuda()).sum(), leaves)
    torch.cuda.synchronize()
    got = [t.detach().float().cpu() for t in (z, *grads)]

    ref_leaves = [t.clone().requires_grad_() for t in (q, k, v)]
    z_r = oracle.vmonarch_attention(*ref_leaves, m, b, c["iters"], recompute_tokens=c["r"])
    g_r = torch.autograd.grad((z_r * dz).sum(), ref_leaves)
    check_vm(got, [z_r.detach(), *(g.detach() for g in g_r)])


def fp8_draw(seed):
    r = random.Random(20_000 + seed)
    m = r.randint(2, 40)
    b = r.choice([64, 100, 128, 129, 200, 256, 300])
    N = m * b
    return dict(B=r.choice([1, 2]), H=r.choice([1, 2]), m=m, b=b, iters=r.choice([1, 2, 3]),
                r=r.choice([0, b, r.randint(1, N)]), token_major=r.random() < 0.3)


FP8_CASES = [fp8_draw(s) for s in range(12)]


@pytest.mark.parametrize("case", FP8_CASES, ids=[f"s{i}-" + "-".join(f"{k}{v}" for k, v in c.items())
                                                 for i, c in enumerate(FP8_CASES)])
def test_vmonarch_fp8_sweep(case):
    """The opt-in e4m3 R step on seeded grids (D = 128, bf16): z against the oracle whose R step
    emulates the e4m3 kernels, and against the exact oracle no further than that emulation is
    (its mean-abs error x 1.5 + 5e-4); gradients against the exact oracle (bounds of test_fp8_gpu)."""
    from test_fp8_gpu import e4m3_oracle_z, run_cuda_fp8
    from test_vmonarch_gpu import run_oracle
    c = case
    B, H, m, b = c["B"], c["H"], c["m"], c["b"]
    gen = torch.Generator().manual_seed(3000 + m * b)
    q, k, v = (torch.randn(B, H, m * b, 128, generator=gen).bfloat16().float() for _ in range(3))
    dz = torch.randn(B, H, m * b, 128, generator=gen)
    got = run_cuda_fp8(q, k, v, dz, m, b, c["iters"], c["r"], c["token_major"])
    exact = run_oracle(q, k, v, dz, m, b, c["iters"], c["r"])
    z8 = e4m3_oracle_z(q, k, v, m, b, c["iters"], c["r"])
    err = (got[0] - z8).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max().item(), err.mean().item())
    own = (z8 - exact[0]).abs().mean().item()  # the e4m3 arithmetic's own error at this shape
    assert (got[0] - exact[0]).abs().mean() <= 1.5 * own + 5e-4, own
    for g, g_r in zip(got[1:], exact[1:]):
        assert (g - g_r).abs().max() <= 5e-2
