"""FP8 (e4m3) R step, an opt-in B200 extension with no reference counterpart, against the fp32 oracle.

* vmb_quant_e4m3 against torch's float8_e4m3fn conversion (round to nearest even), including the
  saturation at +-448 and token-major sources.
* The e4m3 FlashEntropyAttention forward in both R-step forms (values aliasing keys, without and
  with the 128-wide second value tensor) against an fp32 emulation of its arithmetic on the same
  e4m3 inputs: P = 2^(x - m_ref) with the kernel's reference max (the first key tile's, which the
  test checks no later tile passes by the rescale threshold), rounded to e4m3, o = P W / l with l
  the unrounded sum, then rounded to o's type. o within max-abs 1e-2 / mean-abs 2e-5 of it (the
  kernel's exp2 may round a p to the neighbouring e4m3 value), the log2-domain LSE and the entropy
  within 1e-3. Against the exact fp32 attention on the same inputs, o carries the e4m3 rounding of
  P: mean-abs <= 4e-3.
* VMonarch with fp8_r_step. Its z against the fp32 oracle whose R step is replaced by the same
  e4m3 emulation (the kernel's arithmetic: q rounded unscaled with the scale folded into the
  scores, u, k, [k | v] and P rounded to e4m3), at the north-star absolute bounds (z max-abs
  2e-2, mean-abs 2e-3): ragged grids, one to three iterations, recompute lengths, token-major
  inputs. (The emulation rounds fp32 intermediates where the kernels round 16-bit ones, so an
  element of u can land on the neighbouring e4m3 value: no tighter elementwise match exists.) The gradients (the 16-bit backward at the e4m3 forward's statistics) against
  the exact oracle's, max-abs 5e-2 and max-rel 0.1. Accuracy against the exact oracle: at the
  README shape, config 2 and on four heads of the dit14b layer the north-star bounds of the 16-bit
  path hold (z max-abs 2e-2 / mean-abs 2e-3, max-rel 3e-2; gradients 5e-2); on the small ragged
  grids below the e4m3 rounding of P (steps of 6 %) averages over few keys (one iteration, or
  ~100 keys per grid row) and z is held to mean-abs 4e-3 and to 1.5 x the emulation's own
  mean-abs error + 5e-4 (the CPU emulation gives max-rel up to 0.08 there).
"""
import pytest
import torch

import oracle
from oracle import vmonarch as oracle_vm
from conftest import max_rel_err
from test_fullsize_gpu import _layer_with_checked_heads
from test_vmonarch_gpu import check as check_vm
from test_vmonarch_gpu import run_oracle
from vmonarch_b200 import ops, vmonarch_attention
from vmonarch_b200.configs import WORKLOADS

pytestmark = pytest.mark.gpu

E4 = torch.float8_e4m3fn
LOG2E = 1.4426950408889634


def test_quant_e4m3_matches_torch_conversion():
    gen = torch.Generator().manual_seed(3)
    x = (torch.randn(2, 3, 200, 128, generator=gen) * 4).bfloat16()
    x[0, 0, 0, :8] = torch.tensor([0.0, -0.0, 1e-4, -3e-3, 447.0, 460.0, -1000.0, 2.0 ** -9])
    got = ops.quant_e4m3(x.cuda())
    torch.cuda.synchronize()
    ref = x.float().clamp(-448, 448).to(E4)  # saturation at the largest finite value, then RNE
    assert got.dtype == E4 and got.shape == x.shape
    assert torch.equal(got.cpu().view(torch.uint8), ref.view(torch.uint8))
    # a token-major source (B, N, H, D) seen as (B, H, N, D), and a scale
    tm = x.transpose(1, 2).contiguous().transpose(1, 2).cuda()
    got2 = ops.quant_e4m3(tm, scale=0.25)
    ref2 = (x.float() * 0.25).clamp(-448, 448).to(E4)
    assert got2.is_contiguous() and torch.equal(got2.cpu().view(torch.uint8), ref2.view(torch.uint8))


@pytest.mark.parametrize("b", [100, 257, 1560])
@pytest.mark.parametrize("with_v2", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fea_e4m3_forward(b, with_v2, dtype):
    # R-step batch: B = 1, H = 2, m = 3 grid rows of b tokens; keys double as values ([K | V2] with v2)
    gen = torch.Generator().manual_seed(b + 7 * with_v2)
    shape = (1, 2, 3, b, 128)
    q, k, v = (torch.randn(*shape, generator=gen) for _ in range(3))
    q8, k8, v8 = (ops.quant_e4m3(t.to(dtype).cuda()) for t in (q, k, v))
    dw = 256 if with_v2 else 128
    o = torch.empty(*shape[:-1], dw, device="cuda", dtype=dtype)
    lse = torch.empty(shape[:-1], device="cuda")
    ent = torch.empty(shape[:-1], device="cuda")
    scale = 128 ** -0.5
    ops.fea_fwd(q8, k8, k8, o, lse, ent, scale, v2=v8 if with_v2 else None)
    torch.cuda.synchronize()

    qf, kf, vf = (t.float().cuda() for t in (q8, k8, v8))
    w = torch.cat([kf, vf], -1) if with_v2 else kf
    x = (qf @ kf.transpose(-1, -2)) * (scale * LOG2E)
    m_ref = x[..., :128].amax(-1, keepdim=True)
    assert (x.amax(-1, keepdim=True) <= m_ref + 8).all()  # no lazy rescale: the emulation is the kernel's
    p = torch.exp2(x - m_ref)
    l = p.sum(-1, keepdim=True)
    o_emul = ((p.to(E4).float() @ w) / l).to(dtype).float()
    err = (o.float() - o_emul).abs()
    assert err.max() <= 1e-2 and err.mean() <= 2e-5, (err.max().item(), err.mean().item())
    o_r, e_r = oracle.entropy_attention(qf, kf, w, scale)
    assert (o.float() - o_r).abs().mean() <= 4e-3
    lse_r = (m_ref + torch.log2(l)).squeeze(-1)
    assert (lse - lse_r).abs().max() <= 1e-3 * lse_r.abs().max().clamp_min(1.0)
    assert (ent - e_r).abs().max() <= 1e-3 * max(1.0, e_r.abs().max().item())


def test_fea_e4m3_rejects_other_forms():
    q8 = ops.quant_e4m3(torch.randn(2, 64, 128, device="cuda", dtype=torch.bfloat16))
    k8 = ops.quant_e4m3(torch.randn(2, 64, 128, device="cuda", dtype=torch.bfloat16))
    v8 = ops.quant_e4m3(torch.randn(2, 64, 128, device="cuda", dtype=torch.bfloat16))
    o = torch.empty(2, 64, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="e4m3"):  # separate values (VMonarchError): not an R-step form
        ops.fea_fwd(q8, k8, v8, o, None, None, 0.1)
    with pytest.raises(AssertionError, match="e4m3"):  # mixed operand types
        ops.fea_fwd(q8, k8.float().bfloat16(), k8, o, None, None, 0.1)


def run_cuda_fp8(q, k, v, dz, m, b, iters, r, token_major=False):
    def place(t):
        t = t.cuda().bfloat16()
        return t.transpose(1, 2).contiguous().transpose(1, 2) if token_major else t
    leaves = [place(t).requires_grad_() for t in (q, k, v)]
    z = vmonarch_attention(*leaves, m, b, iters, recompute_tokens=r, fp8_r_step=True)
    grads = torch.autograd.grad((z.float() * dz.cuda()).sum(), leaves)
    torch.cuda.synchronize()
    return [t.detach().float().cpu() for t in (z, *grads)]


class E4m3RStep:
    """The oracle's R step (sm_scale 1, the first call's u = q * scale) with the fp8 kernel's
    arithmetic: the first call rounds q itself and folds the scale into the scores; u, k, the
    values and P = 2^(x - m_ref) (m_ref: the first key tile's max) are rounded to e4m3, l and the
    entropy use the unrounded p."""

    def __init__(self, scale):
        self.scale, self.calls = scale, 0

    def __call__(self, u, kg, w):
        sm = 1.0
        if self.calls == 0:
            u, sm = u / self.scale, self.scale
        self.calls += 1
        r8 = lambda t: t.clamp(-448, 448).to(E4).float()  # noqa: E731
        x = (r8(u) @ r8(kg).transpose(-1, -2)) * (sm * LOG2E)
        m_ref = x[..., :128].amax(-1, keepdim=True)
        p = torch.exp2(x - m_ref)
        l = p.sum(-1, keepdim=True)
        ent = (torch.log2(l) - (p * (x - m_ref)).sum(-1, keepdim=True) / l).squeeze(-1) / LOG2E
        return (r8(p) @ r8(w)) / l, ent


def e4m3_oracle_z(q, k, v, m, b, iters, r):
    orig = oracle_vm.r_step
    oracle_vm.r_step = E4m3RStep(q.size(-1) ** -0.5)
    try:
        with torch.no_grad():
            return oracle.vmonarch_attention(q, k, v, m, b, iters, recompute_tokens=r)
    finally:
        oracle_vm.r_step = orig


@pytest.mark.parametrize("B, H, m, b, iters, r, token_major, north_star", [
    (1, 2, 4, 256, 2, 256, False, True),    # the README shape at D = 128
    (2, 4, 16, 256, 2, 256, False, True),   # config 2
    (1, 2, 8, 100, 3, 100, False, False),   # three iterations, one ragged key tile per grid row
    (1, 1, 5, 257, 1, 300, False, False),   # one iteration, recompute past the first grid row
    (2, 2, 6, 129, 2, 0, True, False),      # token-major caller tensors, no recompute
])
def test_vmonarch_fp8_r_step(B, H, m, b, iters, r, token_major, north_star):
    gen = torch.Generator().manual_seed(m * b + iters)
    q, k, v = (torch.randn(B, H, m * b, 128, generator=gen).bfloat16().float() for _ in range(3))
    dz = torch.randn(B, H, m * b, 128, generator=gen)
    got = run_cuda_fp8(q, k, v, dz, m, b, iters, r, token_major)
    exact = run_oracle(q, k, v, dz, m, b, iters, r)
    z, z8 = got[0], e4m3_oracle_z(q, k, v, m, b, iters, r)
    err = (z - z8).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
    for g, g_r in zip(got[1:], exact[1:]):
        assert (g - g_r).abs().max() <= 5e-2 and max_rel_err(g, g_r) <= 0.1
    if north_star:
        check_vm(got, exact)
    else:  # no further from the exact oracle than the e4m3 arithmetic itself is
        own = (z8 - exact[0]).abs().mean().item()
        assert (z - exact[0]).abs().mean() <= min(4e-3, 1.5 * own + 5e-4), own


def test_vmonarch_fp8_dit14b_four_heads():
    """The dit14b layer (40 heads) with fp8 R steps; four heads against the oracle on the GPU."""
    w = WORKLOADS["dit14b"]
    heads = (0, 13, 26, 39)
    q, k, v, dz = _layer_with_checked_heads(w, heads, seed=5)
    leaves = [t.requires_grad_() for t in (q, k, v)]
    z = vmonarch_attention(*leaves, w.m, w.b, w.iters, recompute_tokens=w.recompute, fp8_r_step=True)
    grads = torch.autograd.grad(z, leaves, dz)
    torch.cuda.synchronize()
    assert torch.isfinite(z.float()).all() and all(torch.isfinite(g.float()).all() for g in grads)
    for h in heads:
        ref_leaves = [t.detach()[:, h:h + 1].float().requires_grad_() for t in (q, k, v)]
        z_r = oracle.vmonarch_attention(*ref_leaves, w.m, w.b, w.iters, recompute_tokens=w.recompute)
        g_r = torch.autograd.grad(z_r, ref_leaves, dz[:, h:h + 1].float())
        err = (z[:, h:h + 1].float() - z_r).abs()
        assert err.max() <= 2e-2 and err.mean() <= 2e-3, (h, err.max().item(), err.mean().item())
        for g, gr in zip(grads, g_r):
            gerr = (g[:, h:h + 1].float() - gr).abs().max().item()
            assert gerr <= max(5e-2, 8e-3 * gr.abs().max().item()), (h, gerr)
        del ref_leaves, z_r, g_r
        torch.cuda.empty_cache()


def test_vmonarch_fp8_needs_d128():
    q = torch.randn(1, 1, 4 * 64, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError, match="fp8_r_step"):
        vmonarch_attention(q, q, q, 4, 64, 2, fp8_r_step=True)
