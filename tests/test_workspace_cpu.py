"""The backward's workspace bound (vmonarch_b200.ops.bwd_plan) on the host: sizes come from the C ABI's
workspace queries, which need no GPU. The preferred workspace of the last VMonarch R step and of the
exact recompute holds a dS^T buffer (2 bytes per query x key); above the bound the call is split
over its batch, or falls back to the minimal workspace when no chunk keeps that buffer."""
import ctypes

import pytest
import torch

from vmonarch_b200 import _native as N
from vmonarch_b200 import ops


def _args(batch, n_q, n_kv, dv, v_is_k, grad_mode=0):
    a = N.FeaBwdArgs()
    a.batch, a.n_q, a.n_kv, a.d, a.dv = batch, n_q, n_kv, 128, dv
    a.dv1 = 128
    a.v_is_k = int(v_is_k)
    a.grad_mode = grad_mode
    a.q_bs = a.k_bs = a.v_bs = n_q * 128
    return a


@pytest.fixture
def limit():
    old = ops.workspace_limit()
    yield ops.set_workspace_limit
    ops.set_workspace_limit(old)


def test_default_bound_keeps_the_14b_layer_in_one_call(limit):
    last_r = _args(840, 1560, 1560, 256, True, grad_mode=2)
    pref = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(last_r))
    assert pref > N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(last_r))  # dS^T route
    assert ops.bwd_plan(last_r) == (840, pref)
    recompute = _args(40, 1560, 32760, 128, False, grad_mode=3)
    assert ops.bwd_plan(recompute)[0] == 40


def test_720p_layer_is_chunked_under_the_bound(limit):
    limit(16 << 30)
    for a in (_args(1280, 3600, 3600, 256, True, grad_mode=2), _args(40, 3600, 115200, 128, False, grad_mode=3)):
        pref = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a))
        assert pref > 16 << 30
        chunk, nbytes = ops.bwd_plan(a)
        assert chunk < a.batch and nbytes <= 16 << 30
        b = _args(chunk, a.n_q, a.n_kv, a.dv, a.v_is_k, a.grad_mode)
        assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(b)) == nbytes
        assert nbytes > N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(b))  # still the dS^T route


def test_bound_below_any_useful_chunk_uses_the_minimal_workspace(limit):
    a = _args(40, 3600, 115200, 128, False, grad_mode=3)
    limit(64 << 20)  # chunks of dS^T this small would leave too few query tiles for its GEMM
    assert ops.bwd_plan(a) == (40, N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a)))


def test_chunks_follow_the_middle_batch_dimension(limit):
    # VMonarch's last R step in (B, H, m) batch form: chunks are whole heads (m grid rows each) and
    # never cross a batch entry
    a = _args(2 * 40 * 32, 3600, 3600, 256, True, grad_mode=2)
    limit(16 << 30)
    chunk, nbytes = ops.bwd_plan(a, unit=32, group=40 * 32)
    assert chunk % 32 == 0 and chunk <= 40 * 32 and nbytes <= 16 << 30


def test_token_major_views():
    # a (B, N, H, D) buffer seen as (B, H, N, D): the layout the header documents
    B, H, m, b, D = 2, 5, 3, 16, 128
    N_ = m * b
    base = torch.empty(B, N_, H, D, dtype=torch.bfloat16)
    q = base.transpose(1, 2)
    assert ops.viewable(q) and not q.is_contiguous()
    # FlashEntropyAttention over B * H sequences: (n1, n2) = (H, B)
    v = ops._view(q, 2)
    assert (v.row, v.s1, v.s2, v.s3) == (H * D, D, N_ * H * D, 0) and ops._split(q.shape[:-2]) == (H, B)
    # the R step over B * H * m grid rows of b tokens: (n1, n2) = (m, H)
    g = q.unflatten(2, (m, b))
    v = ops._view(g, 3)
    assert (v.row, v.s1, v.s2, v.s3) == (H * D, b * H * D, D, N_ * H * D) and ops._split(g.shape[:-2]) == (m, H)
    # element (s, r, c) of the view formula == torch's indexing
    for s_ in (0, 7, B * H * m - 1):
        c1, c2, c3 = s_ % m, s_ // m % H, s_ // (m * H)
        r = 5
        off = r * v.row + c1 * v.s1 + c2 * v.s2 + c3 * v.s3
        assert g[c3, c2, c1, r].data_ptr() == base.data_ptr() + 2 * off


def test_backward_args_of_a_chunk_slice():
    # the arguments of chunk (heads 2..3 of batch entry 1) point at that slice's first element, with
    # statistics rows of those sequences
    B, H, m, b, D = 2, 4, 3, 16, 128
    tm = lambda c: torch.empty(B, m * b, H, c, dtype=torch.bfloat16).transpose(1, 2).unflatten(2, (m, b))  # noqa: E731
    t = dict(q=tm(D), k=tm(D), v=None, o=torch.empty(B, H, m, b, 2 * D, dtype=torch.bfloat16),
             lse=torch.empty(B * H * m * b), grad_q=torch.empty(B, H, m, b, D))
    t["v"] = t["k"]
    idx = (1, slice(2, 4))
    sub = {n: (x.view(B, H, m, b)[idx].reshape(-1) if n == "lse" else x[idx]) for n, x in t.items()}
    a, lay = ops.bwd_args(sub, 1.0, 2, True, True)
    assert a.batch == 2 * m and (lay.n1, lay.n2) == (m, 2)
    assert a.q == t["q"][1, 2].data_ptr() and a.o == t["o"][1, 2].data_ptr()
    assert a.lse == t["lse"].data_ptr() + 4 * ((1 * H + 2) * m * b)
    assert (lay.q.row, lay.q.s1, lay.q.s2) == (H * D, b * H * D, D)
