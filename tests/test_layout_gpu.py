"""Token-major callers: the reference's Video-DiT caller holds tokens as (B, N, H, D)
(README.md:74-76) and reaches the attention through a transpose to (B, H, N, D). Those transposed
views are read and written in place through strided layouts (include/vmonarch_b200.h, ABI 6): no
copy of q, k, v, o / z or the gradients is made, the outputs come back token-major, and the results
are exactly those of dense inputs (same kernels, same summation order) and within the parity
tolerances of the fp32 oracle."""
import ctypes

import pytest
import torch

import oracle
from conftest import max_rel_err
from vmonarch_b200 import _native as N
from vmonarch_b200 import flash_entropy_attention, ops, vmonarch_attention

pytestmark = pytest.mark.gpu


def token_major(x: torch.Tensor) -> torch.Tensor:
    """The (B, H, N, C) tensor `x` stored as a (B, N, H, C) buffer and seen through transpose(1, 2)."""
    return x.transpose(1, 2).contiguous().transpose(1, 2)


def packed_qkv(q, k, v):
    """q, k, v stored in one (B, N, 3, H, D) buffer, as a fused QKV projection writes them."""
    buf = torch.stack([t.transpose(1, 2) for t in (q, k, v)], dim=2).contiguous()
    return [buf[:, :, i].transpose(1, 2) for i in range(3)]


def is_token_major(x: torch.Tensor) -> bool:
    return x.transpose(1, 2).is_contiguous()


@pytest.mark.parametrize("layout", ["token_major", "packed_qkv"])
@pytest.mark.parametrize("B, H, N, D", [(1, 6, 1000, 128), (2, 3, 333, 128), (2, 3, 333, 64)])
def test_fea_token_major_in_place(layout, B, H, N, D):
    gen = torch.Generator().manual_seed(N + H)
    q, k, v, do = (torch.randn(B, H, N, D, generator=gen).bfloat16().cuda() for _ in range(4))
    de = torch.randn(B, H, N, generator=gen).cuda()

    def run(q, k, v, do):
        leaves = [t.detach().requires_grad_() for t in (q, k, v)]
        o, e = flash_entropy_attention(*leaves)
        return (o, e, *torch.autograd.grad((o, e), leaves, (do, de)))

    dense = run(q, k, v, do)
    if layout == "packed_qkv":
        tq, tk, tv = packed_qkv(q, k, v)
    else:
        tq, tk, tv = token_major(q), token_major(k), token_major(v)
    snap = [t.clone() for t in (tq, tk, tv)]
    got = run(tq, tk, tv, token_major(do))
    torch.cuda.synchronize()
    assert is_token_major(got[0])  # o in the caller's layout
    for t, s in zip((tq, tk, tv), snap):
        assert torch.equal(t, s)  # inputs untouched
    for g, r in zip(got, dense):
        assert torch.equal(g, r)
    # and within the parity tolerances of the fp32 oracle (one head)
    h = H - 1
    leaves = [t[0, h].float().cpu().requires_grad_() for t in (q, k, v)]
    o_r, e_r = oracle.entropy_attention(*leaves, D ** -0.5)
    g_r = torch.autograd.grad((o_r * do[0, h].float().cpu()).sum() + (e_r * de[0, h].cpu()).sum(), leaves)
    o = got[0][0, h].float().cpu()
    assert (o - o_r).abs().max() <= 2e-2 and (o - o_r).abs().mean() <= 2e-3
    assert (got[1][0, h].cpu() - e_r).abs().max() <= 1e-3 * e_r.abs().max()
    for g, r in zip(got[2:], g_r):
        assert max_rel_err(g[0, h].cpu(), r) <= 3e-2


@pytest.mark.parametrize("B, H, m, b, iters, r", [(1, 4, 8, 200, 2, 200), (2, 3, 21, 130, 3, 130), (1, 2, 5, 96, 1, 0)])
def test_vmonarch_token_major_in_place(B, H, m, b, iters, r):
    gen = torch.Generator().manual_seed(m * b + H)
    q, k, v, dz = (torch.randn(B, H, m * b, 128, generator=gen).bfloat16().cuda() for _ in range(4))

    def run(q, k, v, dz):
        leaves = [t.detach().requires_grad_() for t in (q, k, v)]
        z = vmonarch_attention(*leaves, m, b, iters, recompute_tokens=r)
        return (z, *torch.autograd.grad(z, leaves, dz))

    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        dense = run(q, k, v, dz)
        got = run(token_major(q), token_major(k), token_major(v), token_major(dz))
        torch.cuda.synchronize()
    finally:
        torch.use_deterministic_algorithms(False)
    assert all(is_token_major(t) for t in got)  # z and the gradients in the caller's layout
    for g, d in zip(got, dense):
        assert torch.equal(g, d)
    # one head against the fp32 oracle, with the north-star bounds
    sl = (slice(B - 1, B), slice(H - 1, H))
    leaves = [t[sl].float().requires_grad_() for t in (q, k, v)]
    z_r = oracle.vmonarch_attention(*leaves, m, b, iters, recompute_tokens=r)
    g_r = torch.autograd.grad(z_r, leaves, dz[sl].float())
    err = (got[0][sl].float() - z_r).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3
    for g, gr in zip(got[1:], g_r):
        assert (g[sl].float() - gr).abs().max() <= max(5e-2, 8e-3 * gr.abs().max().item())


def test_fea_forward_token_major_through_the_c_abi():
    # vmb_fea_fwd with a hand-built vmb_fea_layout: (B, N, H, D) buffers, batch index s = b * H + h,
    # (n1, n2) = (H, B), view {row: H * D, s1: D, s2: N * H * D}
    B, H, N_, D = 2, 5, 777, 128
    gen = torch.Generator().manual_seed(3)
    qb, kb, vb = (torch.randn(B, N_, H, D, generator=gen).bfloat16().cuda() for _ in range(3))
    ob = torch.full((B, N_, H, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, H, N_, device="cuda")
    ent = torch.empty(B, H, N_, device="cuda")
    lay = N.FeaLayout()
    lay.n1, lay.n2 = H, B
    for name in ("q", "k", "v", "o"):
        setattr(lay, name, N.View(H * D, D, N_ * H * D, 0))
    a = N.FeaFwdArgs()
    a.q, a.k, a.v, a.o = qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), ob.data_ptr()
    a.lse, a.ent = lse.data_ptr(), ent.data_ptr()
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = B * H, N_, N_, D, D, D
    a.dtype, a.sm_scale = N.VMB_DTYPE_BF16, D ** -0.5
    a.layout = ctypes.pointer(lay)
    nbytes = N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a))
    assert nbytes > 0  # 10 sequences: the key range is split, and the merge kernel writes o through the view
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    N.check(N.lib.vmb_fea_fwd(ctypes.byref(a), N.stream_ptr(qb.device)), "vmb_fea_fwd")
    o_ref = torch.empty(B, H, N_, D, dtype=torch.bfloat16, device="cuda")
    lse_ref, ent_ref = torch.empty_like(lse), torch.empty_like(ent)
    ops.fea_fwd(qb.transpose(1, 2).contiguous(), kb.transpose(1, 2).contiguous(), vb.transpose(1, 2).contiguous(),
                o_ref, lse_ref, ent_ref, D ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(ob.transpose(1, 2), o_ref)
    assert torch.equal(lse, lse_ref) and torch.equal(ent, ent_ref)


def test_strided_cast_through_the_c_abi():
    # vmb_cast_f32_view: an fp32 (B, H, N, D) accumulator into a token-major bf16 gradient
    B, H, N_, D = 2, 3, 100, 128
    src = torch.randn(B, H, N_, D, device="cuda")
    dst = torch.zeros(B, N_, H, D, dtype=torch.bfloat16, device="cuda")
    sv, dv = N.View(D, N_ * D, H * N_ * D, 0), N.View(H * D, D, N_ * H * D, 0)
    N.check(N.lib.vmb_cast_f32_view(src.data_ptr(), ctypes.byref(sv), dst.data_ptr(), ctypes.byref(dv), H, B, B * H,
                                    N_, D, N.VMB_DTYPE_BF16, N.stream_ptr(src.device)), "vmb_cast_f32_view")
    torch.cuda.synchronize()
    assert torch.equal(dst.transpose(1, 2), src.bfloat16())


def test_other_head_dims_fall_back_to_dense_copies():
    # D = 32 runs kernels that take dense tensors only: token-major inputs are copied, results equal
    gen = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, 4, 300, 32, generator=gen).bfloat16().cuda() for _ in range(3))
    o1, e1 = flash_entropy_attention(q, k, v)
    o2, e2 = flash_entropy_attention(token_major(q), token_major(k), token_major(v))
    assert torch.equal(o1, o2) and torch.equal(e1, e2)
