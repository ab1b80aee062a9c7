"""The backward's workspace bound (vmonarch_b200.ops.bwd_plan) on the host: sizes come from the C ABI's
workspace queries, which need no GPU. The preferred workspace of the last VMonarch R step and of the
exact recompute holds a dS^T buffer (2 bytes per query x key); above the bound the call is split
over its batch, or falls back to the minimal workspace when no chunk keeps that buffer."""
import ctypes

import pytest

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
        b = ops._bwd_chunk(a, 0, chunk)
        assert N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(b)) == nbytes
        assert nbytes > N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(b))  # still the dS^T route


def test_bound_below_any_useful_chunk_uses_the_minimal_workspace(limit):
    a = _args(40, 3600, 115200, 128, False, grad_mode=3)
    limit(64 << 20)  # chunks of dS^T this small would leave too few query tiles for its GEMM
    assert ops.bwd_plan(a) == (40, N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a)))


def test_chunk_offsets_every_pointer_by_its_batch_stride():
    a = _args(10, 100, 300, 256, True, grad_mode=1)
    base = 1 << 40
    for i, name in enumerate(("q", "k", "v", "v2", "o", "dout", "lse", "ent", "dent", "delta", "grad_q", "grad_k",
                              "grad_v2", "fin_q")):
        setattr(a, name, base + (i << 32))
    a.v2_bs, a.o_bs, a.do_bs = 300 * 128, 100 * 256, 100 * 256
    a.grad_q_bs, a.grad_k_bs, a.grad_v2_bs, a.fin_q_bs = 100 * 128, 300 * 128, 300 * 128, 100 * 128
    b = ops._bwd_chunk(a, 3, 4)
    assert b.batch == 4 and a.batch == 10
    assert b.q - a.q == 3 * a.q_bs * 2 and b.v2 - a.v2 == 3 * a.v2_bs * 2 and b.dout - a.dout == 3 * a.do_bs * 2
    assert b.lse - a.lse == 3 * 100 * 4 and b.delta - a.delta == 3 * 100 * 4
    assert b.grad_k - a.grad_k == 3 * a.grad_k_bs * 4  # fp32 gradients in grad_mode 1
    assert b.fin_q - a.fin_q == 3 * a.fin_q_bs * 4
    assert b.grad_v is None and b.fin_k is None  # absent pointers stay absent
