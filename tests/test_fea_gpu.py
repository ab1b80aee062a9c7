"""FlashEntropyAttention on the B200 against the fp32 oracle and the reference's golden vectors.

Tolerances, checked both ways:
  reference convention (tests/test_vmonarch.py:22-42): max|x - ref| <= tol * max|ref|, o/e 2e-2,
      gradients 3e-2;
  north-star absolute bounds: o max-abs 2e-2 and mean-abs 2e-3; e within 1e-3 of max|e|;
      gradients max-abs 5e-2 (floored at 8e-3 * max|grad|, the bf16 rounding of large gradients).
"""
import ctypes

import pytest
import torch

import oracle
from conftest import FEA_GOLDEN, load_golden, max_rel_err
from vmonarch_b200 import flash_entropy_attention

pytestmark = pytest.mark.gpu


def run_cuda(q, k, v, do, de, dtype=torch.bfloat16, sm_scale=None):
    leaves = [t.cuda().to(dtype).requires_grad_() for t in (q, k, v)]
    o, e = flash_entropy_attention(*leaves, sm_scale=sm_scale)
    grads = torch.autograd.grad((o.float() * do.cuda()).sum() + (e * de.cuda()).sum(), leaves)
    torch.cuda.synchronize()
    return [t.detach().float().cpu() for t in (o, e, *grads)]


def run_oracle(q, k, v, do, de, sm_scale):
    leaves = [t.float().clone().requires_grad_() for t in (q, k, v)]
    o, e = oracle.entropy_attention(*leaves, sm_scale)
    grads = torch.autograd.grad((o * do).sum() + (e * de).sum(), leaves)
    return [t.detach() for t in (o, e, *grads)]


def check(got, ref):
    o, e, *g = got
    o_r, e_r, *g_r = ref
    assert max_rel_err(o, o_r) <= 2e-2 and max_rel_err(e, e_r) <= 2e-2
    for a, b in zip(g, g_r):
        assert max_rel_err(a, b) <= 3e-2
    assert (o - o_r).abs().max() <= 2e-2 and (o - o_r).abs().mean() <= 2e-3
    # relative to the largest entropy, floored for single-key rows (exactly 0 in the reference;
    # x - m = fma(s, scale, -m) keeps the rounding residual of s * scale, ~1e-8)
    assert (e - e_r).abs().max() <= max(1e-3 * e_r.abs().max().item(), 1e-6)
    for a, b in zip(g, g_r):
        assert (a - b).abs().max() <= max(5e-2, 8e-3 * b.abs().max().item())


@pytest.mark.parametrize("name", FEA_GOLDEN)
def test_fea_against_reference_golden(name):
    g = load_golden(name)
    got = run_cuda(g["q"], g["k"], g["v"], g["do"], g["de"])
    check(got, [g[x] for x in ("o", "e", "dq", "dk", "dv")])


@pytest.mark.parametrize("N", [128, 200, 1024])
@pytest.mark.parametrize("D, Dv", [(64, 64), (128, 128), (64, 128), (128, 256)])
def test_flash_entropy_attention(N, D, Dv):
    # the reference's test matrix (tests/test_vmonarch.py:27-42): B=2, H=3, random dO and dE
    gen = torch.Generator().manual_seed(0)
    q, k = (torch.randn(2, 3, N, D, generator=gen).bfloat16().float() for _ in range(2))
    v = torch.randn(2, 3, N, Dv, generator=gen).bfloat16().float()
    do, de = torch.randn(2, 3, N, Dv, generator=gen), torch.randn(2, 3, N, generator=gen)
    check(run_cuda(q, k, v, do, de), run_oracle(q, k, v, do, de, D ** -0.5))


@pytest.mark.parametrize("N", [100, 300])
@pytest.mark.parametrize("D, Dv", [(16, 16), (16, 64), (32, 32), (32, 256), (256, 256)])
def test_head_dims_16_32_256(N, D, Dv):
    # the remaining head dims the reference accepts (kernel.py:324: D, Dv in {16, ..., 256},
    # Dv % D == 0), on the warp-level MMA kernels with 64-column shared-memory rows
    gen = torch.Generator().manual_seed(N + D + Dv)
    q, k = (torch.randn(2, 3, N, D, generator=gen).bfloat16().float() for _ in range(2))
    v = torch.randn(2, 3, N, Dv, generator=gen).bfloat16().float()
    do, de = torch.randn(2, 3, N, Dv, generator=gen), torch.randn(2, 3, N, generator=gen)
    check(run_cuda(q, k, v, do, de), run_oracle(q, k, v, do, de, D ** -0.5))


@pytest.mark.parametrize("N", [1, 17, 64, 127, 129, 150, 333])
@pytest.mark.parametrize("D", [64, 128])
def test_ragged_and_tiny_sequences(N, D):
    # D = 128 runs the tcgen05 kernels: a last key tile of <= 32 keys (N = 1, 17, 129, 150) goes
    # through the N = 32 MMAs
    gen = torch.Generator().manual_seed(N)
    q, k, v = (torch.randn(1, 5, N, D, generator=gen).bfloat16().float() for _ in range(3))
    do, de = torch.randn(1, 5, N, D, generator=gen), torch.randn(1, 5, N, generator=gen)
    check(run_cuda(q, k, v, do, de), run_oracle(q, k, v, do, de, D ** -0.5))


def test_fp16_and_custom_scale():
    gen = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, 2, 300, 128, generator=gen).half().float() for _ in range(3))
    do, de = torch.randn(1, 2, 300, 128, generator=gen), torch.randn(1, 2, 300, generator=gen)
    got = run_cuda(q, k, v, do, de, dtype=torch.float16, sm_scale=0.05)
    check(got, run_oracle(q, k, v, do, de, 0.05))


@pytest.mark.parametrize("N", [300, 2100])
def test_fp16_values_aliasing_keys(N):
    # fp16, D = 128, V passed as K: the one-stream forward (300 keys on 40 sequences: no split) and
    # the split two-stream one (2100 keys on 2 sequences), then the V-aliasing backward
    H = 40 if N == 300 else 2
    gen = torch.Generator().manual_seed(N + 5)
    q, k = (torch.randn(1, H, N, 128, generator=gen).half().float() for _ in range(2))
    do, de = torch.randn(1, H, N, 128, generator=gen), torch.randn(1, H, N, generator=gen)
    qc, kc = (t.cuda().half().requires_grad_() for t in (q, k))
    o, e = flash_entropy_attention(qc, kc, kc)
    gq, gk = torch.autograd.grad((o.float() * do.cuda()).sum() + (e * de.cuda()).sum(), (qc, kc))
    torch.cuda.synchronize()
    n = min(H, 3)
    got = [t.detach().float().cpu()[:, :n] for t in (o, e, gq, gk)]
    qr, kr = (t[:, :n].clone().requires_grad_() for t in (q, k))
    o_r, e_r = oracle.entropy_attention(qr, kr, kr, 128 ** -0.5)
    gq_r, gk_r = torch.autograd.grad((o_r * do[:, :n]).sum() + (e_r * de[:, :n]).sum(), (qr, kr))
    check(got, [o_r.detach(), e_r.detach(), gq_r, gk_r])


def test_noncontiguous_inputs_and_no_mutation():
    gen = torch.Generator().manual_seed(8)
    base = torch.randn(1, 200, 2, 64, generator=gen).bfloat16().cuda()
    q = base.transpose(1, 2)  # (1, 2, 200, 64) non-contiguous view
    snapshot = base.clone()
    o, e = flash_entropy_attention(q, q, q)
    o2, e2 = flash_entropy_attention(q.contiguous(), q.contiguous(), q.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(base, snapshot)
    assert torch.equal(o, o2) and torch.equal(e, e2)


def test_deterministic_forward():
    gen = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(2, 2, 500, 128, generator=gen).bfloat16().cuda() for _ in range(3))
    a = flash_entropy_attention(q, k, v)
    b = flash_entropy_attention(q, k, v)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("D, Dv", [(128, 128), (128, 256), (64, 64)])
def test_growing_row_max_forces_rescales(D, Dv):
    # Later key tiles score far higher than the first ones, so the running max of many (but not
    # all) rows jumps by more than the lazy-rescale threshold at different tiles: exercises the
    # O / l / h rescale path with rows of one warp disagreeing.
    gen = torch.Generator().manual_seed(21)
    N = 640
    q = torch.randn(1, 2, N, D, generator=gen)
    k = torch.randn(1, 2, N, D, generator=gen)
    boost = torch.linspace(0.0, 3.0, N).view(1, 1, N, 1)
    c = torch.randn(1, 2, 1, D, generator=gen)
    q = (q + 1.5 * c * (torch.rand(1, 2, N, 1, generator=gen) > 0.5)).bfloat16().float()
    k = (k + boost * c).bfloat16().float()
    v = torch.randn(1, 2, N, Dv, generator=gen).bfloat16().float()
    do, de = torch.randn(1, 2, N, Dv, generator=gen), torch.randn(1, 2, N, generator=gen)
    check(run_cuda(q, k, v, do, de), run_oracle(q, k, v, do, de, D ** -0.5))


@pytest.mark.parametrize("Dv, steps", [(128, (320, 704)), (128, (256, 960)), (256, (320, 704))])
def test_row_max_jumps_inside_a_key_tile(Dv, steps):
    # The scores of half the rows jump far past the lazy-rescale threshold at fixed keys: at the
    # second 64-key half of a tile (320, 704), or at a tile start (256, 960). Full tiles after a
    # stream's first take the exponentials against the running reference and redo a half whose
    # max passed it, so this covers the redo in either half, with rows of one warp disagreeing.
    gen = torch.Generator().manual_seed(23)
    N, D = 1152, 128
    q = torch.randn(1, 2, N, D, generator=gen)
    k = torch.randn(1, 2, N, D, generator=gen)
    c = torch.randn(1, 2, 1, D, generator=gen)
    q = (q + 1.5 * c * (torch.rand(1, 2, N, 1, generator=gen) > 0.5)).bfloat16().float()
    for st in steps:
        k[:, :, st:] += 1.5 * c
    k = k.bfloat16().float()
    v = torch.randn(1, 2, N, Dv, generator=gen).bfloat16().float()
    do, de = torch.randn(1, 2, N, Dv, generator=gen), torch.randn(1, 2, N, generator=gen)
    check(run_cuda(q, k, v, do, de), run_oracle(q, k, v, do, de, D ** -0.5))


@pytest.mark.parametrize("copies", [1, 20])
@pytest.mark.parametrize("steps", [(320, 704), (256, 960), (64, 448)])
def test_values_aliasing_keys_with_row_max_jumps(steps, copies):
    # V passed as the same tensor as K with D = 128, two sequences of 1152 keys. Alone (copies = 1)
    # the forward splits the key range and runs the two-stream kernel; repeated 20 times there are
    # too many CTAs for a split, and the one-stream kernel runs (S in 64-key halves, each issued
    # behind P V of the previous tile's same half), whose rescale of O waits for the previous
    # tile's second P V half (a jump in a tile's first half) or for this tile's first (a jump in
    # the second half). Half the rows see the jumps (each ~12 in log2 units, past the threshold of
    # 8), with steps small enough that the values (= keys) stay O(1) for the absolute output bound.
    # The oracle checks the first two sequences.
    from vmonarch_b200 import _native as N_
    gen = torch.Generator().manual_seed(29)
    N, D = 1152, 128
    q = torch.randn(1, 2, N, D, generator=gen)
    k = torch.randn(1, 2, N, D, generator=gen)
    c = torch.randn(1, 2, 1, D, generator=gen)
    q = (q + 1.5 * c * (torch.rand(1, 2, N, 1, generator=gen) > 0.5)).bfloat16().float()
    for st in steps:
        k[:, :, st:] += 0.5 * c
    k = k.bfloat16().float()
    do, de = torch.randn(1, 2, N, D, generator=gen), torch.randn(1, 2, N, generator=gen)

    a = N_.FeaFwdArgs()
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = 2 * copies, N, N, D, D, D
    a.dtype = N_.dtype_code(torch.bfloat16)
    assert (N_.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a)) == 0) == (copies > 1)
    rep = lambda t: t.repeat(1, copies, *([1] * (t.dim() - 2)))  # noqa: E731
    qc, kc = (rep(t).cuda().bfloat16().requires_grad_() for t in (q, k))
    o, e = flash_entropy_attention(qc, kc, kc)
    gq, gk = torch.autograd.grad((o.float() * rep(do).cuda()).sum() + (e * rep(de).cuda()).sum(), (qc, kc))
    torch.cuda.synchronize()
    got = [t.detach().float().cpu()[:, :2] for t in (o, e, gq, gk)]

    qr, kr = (t.float().clone().requires_grad_() for t in (q, k))
    o_r, e_r = oracle.entropy_attention(qr, kr, kr, D ** -0.5)
    gq_r, gk_r = torch.autograd.grad((o_r * do).sum() + (e_r * de).sum(), (qr, kr))
    ref = [o_r.detach(), e_r.detach(), gq_r, gk_r]
    # check() pairs gradients by position: (dq, dk) here, dk holding both the key and value roles
    check(got, ref)


def test_values_aliasing_keys_long_sequence():
    # V passed as K over 2100 keys on two sequences: the forward splits the key range (a workspace
    # is given), which runs the two-stream kernel (two query tiles per CTA, 17 of them here, so the
    # last CTA's second stream runs on a zero-filled tile); with V aliasing K each K slot is freed
    # only after both streams' P V of that key tile. Forward and gradients against the oracle.
    gen = torch.Generator().manual_seed(31)
    N, D = 2100, 128
    q, k = (torch.randn(1, 2, N, D, generator=gen).bfloat16().float() for _ in range(2))
    do, de = torch.randn(1, 2, N, D, generator=gen), torch.randn(1, 2, N, generator=gen)
    qc, kc = (t.cuda().bfloat16().requires_grad_() for t in (q, k))
    o, e = flash_entropy_attention(qc, kc, kc)
    gq, gk = torch.autograd.grad((o.float() * do.cuda()).sum() + (e * de.cuda()).sum(), (qc, kc))
    torch.cuda.synchronize()
    got = [t.detach().float().cpu() for t in (o, e, gq, gk)]
    qr, kr = (t.float().clone().requires_grad_() for t in (q, k))
    o_r, e_r = oracle.entropy_attention(qr, kr, kr, D ** -0.5)
    gq_r, gk_r = torch.autograd.grad((o_r * do).sum() + (e_r * de).sum(), (qr, kr))
    check(got, [o_r.detach(), e_r.detach(), gq_r, gk_r])


def test_values_aliasing_keys_long_unsplit():
    # V passed as K over 2100 keys on 40 sequences: too many CTAs for a key-range split (no forward
    # workspace), so the forward runs the one-stream kernel over 17 key tiles, the last one 52 keys
    # wide (its second S half is not issued). All 40 sequences run on the GPU; the oracle checks
    # the first three, the others only for finite values.
    from vmonarch_b200 import _native as N
    gen = torch.Generator().manual_seed(37)
    H, N_, D, n_chk = 40, 2100, 128, 3
    a = N.FeaFwdArgs()
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = H, N_, N_, D, D, D
    a.dtype = N.dtype_code(torch.bfloat16)
    assert N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a)) == 0
    q, k = (torch.randn(1, H, N_, D, generator=gen).bfloat16().float() for _ in range(2))
    do, de = torch.randn(1, H, N_, D, generator=gen), torch.randn(1, H, N_, generator=gen)
    qc, kc = (t.cuda().bfloat16().requires_grad_() for t in (q, k))
    o, e = flash_entropy_attention(qc, kc, kc)
    gq, gk = torch.autograd.grad((o.float() * do.cuda()).sum() + (e * de.cuda()).sum(), (qc, kc))
    torch.cuda.synchronize()
    got = [t.detach().float().cpu() for t in (o, e, gq, gk)]
    assert all(torch.isfinite(t).all() for t in got)
    qr, kr = (t[:, :n_chk].clone().requires_grad_() for t in (q, k))
    o_r, e_r = oracle.entropy_attention(qr, kr, kr, D ** -0.5)
    gq_r, gk_r = torch.autograd.grad((o_r * do[:, :n_chk]).sum() + (e_r * de[:, :n_chk]).sum(), (qr, kr))
    check([t[:, :n_chk] for t in got], [o_r.detach(), e_r.detach(), gq_r, gk_r])


def test_split_key_range_backward_matches_and_is_deterministic(monkeypatch):
    # Few query tiles over a long key range: in fp32-accumulate mode the dQ kernel splits the key
    # range over several CTAs (partial tiles summed in a fixed order). The workspace is held to the
    # minimal size (the split's partial tiles, no dS^T), so the split runs whatever route the
    # preferred size would allow. Check it against the unsplit 16-bit mode and that two runs are
    # bitwise identical.
    from vmonarch_b200 import _native as N, ops
    import ctypes
    gen = torch.Generator().manual_seed(21)
    B, nq, nk, D = 2, 128, 4096, 128
    q = torch.randn(B, nq, D, generator=gen).bfloat16().cuda()
    k, v = (torch.randn(B, nk, D, generator=gen).bfloat16().cuda() for _ in range(2))
    do = torch.randn(B, nq, D, generator=gen).bfloat16().cuda()
    de = torch.randn(B, nq, generator=gen).cuda()
    sm = D ** -0.5
    o = torch.empty_like(q)
    lse, ent = torch.empty(B, nq, device="cuda"), torch.empty(B, nq, device="cuda")
    ops.fea_fwd(q, k, v, o, lse, ent, sm)
    a = N.FeaBwdArgs()
    a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1, a.grad_mode = B, nq, nk, D, D, D, 1
    least = N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a))
    assert least > 3 * B * 128 * 4 * 2  # partial tiles present
    monkeypatch.setattr(N.lib, "vmb_fea_bwd_workspace_bytes", lambda args: least)

    ref = [torch.empty_like(t) for t in (q, k, v)]
    ops.fea_bwd(q, k, v, o, do, lse, *ref, sm, ent=ent, dent=de, grad_mode=0)
    runs = []
    for _ in range(2):
        acc = [torch.zeros(t.shape, device="cuda") for t in (q, k, v)]
        ops.fea_bwd(q, k, v, o, do, lse, *acc, sm, ent=ent, dent=de, grad_mode=1)
        runs.append(acc)
    torch.cuda.synchronize()
    for g, r in zip(runs[0], ref):
        assert max_rel_err(g, r.float()) <= 1e-2
    for g0, g1 in zip(*runs):
        assert torch.equal(g0, g1)


@pytest.mark.parametrize("D", [128, 64, 32])
def test_grad_mode_overwrite_equals_add_into_zeros(D):
    # grad_mode 2 overwrites fp32 gradient buffers (here pre-filled with NaN); it must give exactly
    # what grad_mode 1 adds into zero-filled ones. D = 128 and 64 run the tcgen05 kernels (64: over
    # 64-column tensor maps), D = 32 mma.sync.
    from vmonarch_b200 import ops
    gen = torch.Generator().manual_seed(5)
    B, n = 3, 300
    q, k, v, do = (torch.randn(B, n, D, generator=gen).bfloat16().cuda() for _ in range(4))
    de = torch.randn(B, n, generator=gen).cuda()
    o = torch.empty_like(q)
    lse, ent = torch.empty(B, n, device="cuda"), torch.empty(B, n, device="cuda")
    ops.fea_fwd(q, k, v, o, lse, ent, D ** -0.5)
    add = [torch.zeros(t.shape, device="cuda") for t in (q, k, v)]
    ops.fea_bwd(q, k, v, o, do, lse, *add, D ** -0.5, ent=ent, dent=de, grad_mode=1)
    put = [torch.full(t.shape, float("nan"), device="cuda") for t in (q, k, v)]
    ops.fea_bwd(q, k, v, o, do, lse, *put, D ** -0.5, ent=ent, dent=de, grad_mode=2)
    torch.cuda.synchronize()
    for a, p in zip(add, put):
        assert torch.isfinite(p).all()
        if D in (64, 128):
            assert torch.equal(a, p)
        else:  # the mma.sync kernels add dQ with atomics: the summation order varies run to run
            torch.testing.assert_close(p, a, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n", [300, 1560, 4096])
@pytest.mark.parametrize("mode", [1, 2])
def test_fused_dq_backward_v_is_k(n, mode):
    # V aliasing K with Dv = D = 128 and <= 32 key tiles (the first VMonarch R step): dQ is formed
    # inside the dK kernel and reduce-added into fp32. Check it against the deterministic two-kernel
    # path, against the fp32 oracle (k in both roles), and the overwrite mode over NaN-filled buffers.
    from vmonarch_b200 import ops
    gen = torch.Generator().manual_seed(n + mode)
    B, D = 3, 128
    q, k, do = (torch.randn(B, n, D, generator=gen).bfloat16() for _ in range(3))
    de = torch.randn(B, n, generator=gen) * 0.1
    sm = D ** -0.5
    qc, kc, doc, dec = q.cuda(), k.cuda(), do.cuda(), de.cuda()
    o = torch.empty_like(qc)
    lse, ent = torch.empty(B, n, device="cuda"), torch.empty(B, n, device="cuda")
    ops.fea_fwd(qc, kc, kc, o, lse, ent, sm)
    out = {}
    for det in (True, False):
        fill = float("nan") if mode == 2 else 0.0
        gq, gk = (torch.full((B, n, D), fill, device="cuda") for _ in range(2))
        ops.fea_bwd(qc, kc, kc, o, doc, lse, gq, gk, None, sm, ent=ent, dent=dec, grad_mode=mode, v_is_k=True,
                    deterministic=det)
        out[det] = (gq.cpu(), gk.cpu())
    torch.cuda.synchronize()
    for g_f, g_d in zip(out[False], out[True]):
        assert torch.isfinite(g_f).all()
        assert max_rel_err(g_f, g_d) <= 1e-3
    if n == 300:
        ql, kl = q.float().requires_grad_(), k.float().requires_grad_()
        o_r, e_r = oracle.entropy_attention(ql, kl, kl, sm)
        gq_r, gk_r = torch.autograd.grad((o_r * do.float()).sum() + (e_r * de).sum(), (ql, kl))
        for g, r in zip(out[False], (gq_r, gk_r)):
            assert max_rel_err(g, r) <= 3e-2
            assert (g - r).abs().max() <= max(5e-2, 8e-3 * r.abs().max().item())


@pytest.mark.parametrize("n", [300, 1560])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_backward_keys_as_values_with_v2(n, mode):
    # The last VMonarch R step: values [K | V2] (Dv = 256) with V aliasing K. Gradients of q, of k
    # (key and value roles summed) and of v2 against the fp32 oracle, in every write mode.
    from vmonarch_b200 import ops
    gen = torch.Generator().manual_seed(7 * n + mode)
    B, D = 2, 128
    q, k, v2 = (torch.randn(B, n, D, generator=gen).bfloat16() for _ in range(3))
    do = torch.randn(B, n, 2 * D, generator=gen).bfloat16()
    de = torch.randn(B, n, generator=gen) * 0.1
    sm = D ** -0.5
    qc, kc, v2c, doc, dec = q.cuda(), k.cuda(), v2.cuda(), do.cuda(), de.cuda()
    o = torch.empty(B, n, 2 * D, dtype=torch.bfloat16, device="cuda")
    lse, ent = torch.empty(B, n, device="cuda"), torch.empty(B, n, device="cuda")
    ops.fea_fwd(qc, kc, kc, o, lse, ent, sm, v2=v2c)
    if mode == 0:
        gq, gk, gv2 = (torch.empty(B, n, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    else:
        fill = float("nan") if mode == 2 else 0.0
        gq, gk, gv2 = (torch.full((B, n, D), fill, device="cuda") for _ in range(3))
    ops.fea_bwd(qc, kc, kc, o, doc, lse, gq, gk, None, sm, ent=ent, dent=dec, v2=v2c, grad_v2=gv2, grad_mode=mode,
                v_is_k=True)
    torch.cuda.synchronize()
    ql, kl, vl = q.float().requires_grad_(), k.float().requires_grad_(), v2.float().requires_grad_()
    o_r, e_r = oracle.entropy_attention(ql, kl, torch.cat([kl, vl], -1), sm)
    refs = torch.autograd.grad((o_r * do.float()).sum() + (e_r * de).sum(), (ql, kl, vl))
    for g, r in zip((gq, gk, gv2), refs):
        g = g.float().cpu()
        assert torch.isfinite(g).all()
        assert max_rel_err(g, r) <= 3e-2
        assert (g - r).abs().max() <= max(5e-2, 8e-3 * r.abs().max().item())


@pytest.mark.parametrize("case", ["plain", "split", "v2", "d64", "split64", "d32"])
def test_grad_mode_finalize_equals_add_then_cast(case):
    # grad_mode 3 writes 16-bit gradients as fp32 accumulator + this call's gradient; it must equal
    # adding into the accumulators (grad_mode 1) and converting afterwards, bit for bit.
    from vmonarch_b200 import ops
    gen = torch.Generator().manual_seed(hash(case) % 1000)
    B, nq, nk, D = {"plain": (3, 300, 300, 128), "split": (2, 128, 4096, 128), "v2": (2, 300, 300, 128),
                    "d64": (2, 200, 200, 64), "split64": (2, 128, 4096, 64), "d32": (2, 200, 200, 32)}[case]
    q = torch.randn(B, nq, D, generator=gen).bfloat16().cuda()
    k, v = (torch.randn(B, nk, D, generator=gen).bfloat16().cuda() for _ in range(2))
    v_is_k, v2 = case == "v2", None
    if v_is_k:
        v, v2 = k, v
    dv_w = 2 * D if v_is_k else D
    do = torch.randn(B, nq, dv_w, generator=gen).bfloat16().cuda()
    sm = D ** -0.5
    o = torch.empty(B, nq, dv_w, dtype=torch.bfloat16, device="cuda")
    lse, ent = torch.empty(B, nq, device="cuda"), torch.empty(B, nq, device="cuda")
    ops.fea_fwd(q, k, v, o, lse, ent, sm, v2=v2)
    shapes = [(B, nq, D), (B, nk, D), (B, nk, D)]
    acc = [torch.randn(s_, generator=gen).cuda() for s_ in shapes]
    add = [a.clone() for a in acc]
    gv = None if v_is_k else add[2]
    ops.fea_bwd(q, k, v, o, do, lse, add[0], add[1], gv, sm, v2=v2, grad_v2=add[2] if v_is_k else None,
                grad_mode=1, v_is_k=v_is_k, deterministic=True)
    ref = [a.bfloat16() for a in add]
    out = [torch.empty(s_, dtype=torch.bfloat16, device="cuda") for s_ in shapes]
    fin = [a.clone() for a in acc]
    ops.fea_bwd(q, k, v, o, do, lse, out[0], out[1], None if v_is_k else out[2], sm, v2=v2,
                grad_v2=out[2] if v_is_k else None, grad_mode=3, v_is_k=v_is_k, deterministic=True, fin_q=fin[0],
                fin_k=fin[1], fin_v=None if v_is_k else fin[2], fin_v2=fin[2] if v_is_k else None)
    torch.cuda.synchronize()
    for name, g, r in zip(("dq", "dk", "dv"), out, ref):
        if D in (64, 128):
            assert torch.equal(g, r), name
        else:  # the mma.sync kernels add with atomics: the summation order varies run to run
            torch.testing.assert_close(g.float(), r.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("case", ["last_r", "plain", "long_keys"])
def test_dq_with_and_without_the_ds_workspace(monkeypatch, case):
    # dQ = dS K from the dS^T the dK/dV kernel stores (when the workspace holds it) against the dq
    # kernel that recomputes S and dP (the minimal workspace, as the no-alloc entry point passes):
    # the last VMonarch R step (V aliasing K, V2), a plain dv = 128 call, and the recompute's shape
    # (few queries over a long key range, the fp32 accumulators of grad_mode 1). The preferred
    # workspace holds dS^T in each; both paths must give the same gradients.
    from vmonarch_b200 import _native as N, ops
    gen = torch.Generator().manual_seed(11)
    D = 128
    B, nq, nk = {"last_r": (2, 1560, 1560), "plain": (24, 1560, 2048), "long_keys": (24, 1560, 8192)}[case]
    vk = case == "last_r"
    q = torch.randn(B, nq, D, generator=gen).bfloat16().cuda()
    k, v = (torch.randn(B, nk, D, generator=gen).bfloat16().cuda() for _ in range(2))
    v2 = v if vk else None
    vv = k if vk else v
    dvw = 2 * D if vk else D
    do = torch.randn(B, nq, dvw, generator=gen).bfloat16().cuda()
    sm = D ** -0.5
    o = torch.empty(B, nq, dvw, dtype=torch.bfloat16, device="cuda")
    lse, ent = torch.empty(B, nq, device="cuda"), torch.empty(B, nq, device="cuda")
    ops.fea_fwd(q, k, vv, o, lse, ent, sm, v2=v2)

    def run():
        g = [torch.zeros(B, n_, D, device="cuda") for n_ in (nq, nk, nk)]
        ops.fea_bwd(q, k, vv, o, do, lse, g[0], g[1], None if vk else g[2], sm, v2=v2, grad_v2=g[2] if vk else None,
                    grad_mode=1, v_is_k=vk)
        torch.cuda.synchronize()
        return g

    full = run()
    args = _bwd_args(B, nq, nk, D, vk)
    least = N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(args))
    ds = B * ((nk + 127) // 128 * 128) * ((nq + 63) // 64 * 64) * 2
    preferred = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(args))
    assert preferred >= ds > 0 and least < ds  # the preferred size holds dS^T, the minimal one does not
    monkeypatch.setattr(N.lib, "vmb_fea_bwd_workspace_bytes", lambda a: least)
    small = run()
    for name, a, b in zip(("dq", "dk", "dv"), full, small):
        assert torch.isfinite(a).all() and torch.isfinite(b).all()
        assert max_rel_err(a, b) <= 1e-2, name


def _bwd_args(B, nq, nk, D, vk):
    from vmonarch_b200 import _native as N
    a = N.FeaBwdArgs()
    a.batch, a.n_q, a.n_kv, a.d = B, nq, nk, D
    a.dv, a.dv1, a.grad_mode, a.v_is_k = (2 * D if vk else D), D, 1, int(vk)
    return a


def test_forward_workspace_absent_or_short_runs_unsplit():
    # Through the C ABI, V passed as K over 2100 keys on two sequences: with the workspace the
    # query asks for, the key range splits (two-stream kernel + merge); with no workspace or a
    # shorter one the call still succeeds, unsplit (one-stream kernel). The two unsplit runs are
    # bitwise identical; the split one agrees within float rounding of the merge.
    from vmonarch_b200 import _native as N
    gen = torch.Generator().manual_seed(47)
    B, n, D = 2, 2100, 128
    q, k = (torch.randn(B, n, D, generator=gen).bfloat16().cuda() for _ in range(2))

    def run(ws_bytes):
        o = torch.empty(B, n, D, dtype=torch.bfloat16, device="cuda")
        lse, ent = torch.empty(B, n, device="cuda"), torch.empty(B, n, device="cuda")
        a = N.FeaFwdArgs()
        a.q, a.q_bs, a.k, a.k_bs, a.v, a.v_bs = q.data_ptr(), n * D, k.data_ptr(), n * D, k.data_ptr(), n * D
        a.o, a.o_bs, a.lse, a.ent = o.data_ptr(), n * D, lse.data_ptr(), ent.data_ptr()
        a.batch, a.n_q, a.n_kv, a.d, a.dv, a.dv1 = B, n, n, D, D, D
        a.dtype, a.sm_scale = N.dtype_code(torch.bfloat16), D ** -0.5
        need = N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a))
        ws = None
        if ws_bytes is not None:
            ws = torch.empty(max(need if ws_bytes == "full" else ws_bytes, 16), dtype=torch.uint8, device="cuda")
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel() if ws_bytes == "full" else ws_bytes
        rc = N.lib.vmb_fea_fwd(ctypes.byref(a), N.stream_ptr(q.device))
        assert rc == 0, N.lib.vmb_last_error()
        torch.cuda.synchronize()
        return need, [t.float().cpu() for t in (o, lse, ent)]

    need, full = run("full")
    assert need > 0
    _, none = run(None)
    _, short = run(need // 2)
    for a_, b_ in zip(none, short):
        assert torch.equal(a_, b_)
    o_r, e_r = oracle.entropy_attention(q.float().cpu().unsqueeze(0), k.float().cpu().unsqueeze(0),
                                        k.float().cpu().unsqueeze(0), D ** -0.5)
    for got in (full, none):
        assert (got[0] - o_r[0]).abs().max() <= 2e-2 and max_rel_err(got[2], e_r[0]) <= 2e-2
    # o: at most about one bf16 rounding step apart; lse: fp32 merge rounding
    assert (full[0] - none[0]).abs().max() <= 2e-2 and (full[1] - none[1]).abs().max() <= 1e-4
