"""FlashEntropyAttention: non-causal attention that also returns the row entropy of the attention map.

Drop-in for ``video_monarch_attention.kernel`` (reference ``video_monarch_attention/kernel.py``):
same function name, arguments, return values and assertion behaviour. The forward and backward
run on the hand-written sm_100a kernels behind the C ABI (``include/vmonarch_b200.h``); there is
no padding copy (the reference pads N to a multiple of 128, kernel.py:399-400) and no autotuning.
Token-major inputs ((B, N, H, D) buffers seen as (B, H, N, D) through transpose(1, 2)) are read in
place and o is returned in the same layout.
"""
from __future__ import annotations

import torch

from . import ops

#: dtypes accepted, as in the reference (kernel.py:13)
SUPPORTED_DTYPES = (torch.bfloat16, torch.float16)
#: head dims the reference accepts (kernel.py:324)
_REF_DIMS = {16, 32, 64, 128, 256}


def _check_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """The reference's assertions (kernel.py:322-325, 260) plus the CUDA-device requirement."""
    assert q.dtype in SUPPORTED_DTYPES, f"unsupported dtype {q.dtype}"
    assert k.dtype == q.dtype and v.dtype == q.dtype, "q, k, v must share a dtype"
    assert q.dim() == 4 and k.shape == q.shape and v.shape[:-1] == q.shape[:-1]
    D, Dv = q.shape[-1], v.shape[-1]
    assert D in _REF_DIMS and Dv in _REF_DIMS
    assert Dv % D == 0, "Dv must be a multiple of D"
    assert q.is_cuda and k.device == q.device and v.device == q.device, "vmonarch_b200 needs CUDA tensors"


class _FlashEntropyAttention(torch.autograd.Function):
    """Autograd op; forward (kernel.py:318-358) and backward (kernel.py:360-381) of the reference."""

    @staticmethod
    def forward(ctx, q, k, v, sm_scale, warp_specialize):
        del warp_specialize  # accepted for API compatibility; the kernels are always specialised
        B, H, N, D = q.shape
        Dv = v.shape[-1]
        # dense or token-major ((B, N, H, D) seen through transpose(1, 2)) inputs are read in place
        # by the tcgen05 kernels (D = Dv = 128 or 64); other head dims take dense copies
        strided = (D, Dv) in ((128, 128), (64, 64))
        q, k, v = (t if strided and ops.viewable(t) else t.contiguous() for t in (q, k, v))
        if q.size(1) > 1 and N > 1 and q.stride(1) < q.stride(2):   # token-major: o in the same layout
            o = torch.empty((B, N, H, Dv), device=q.device, dtype=q.dtype).transpose(1, 2)
        else:
            o = torch.empty((B, H, N, Dv), device=q.device, dtype=q.dtype)
        lse = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
        ent = torch.empty((B, H, N), device=q.device, dtype=torch.float32)
        ops.fea_fwd(q, k, v, o, lse, ent, sm_scale)
        ctx.save_for_backward(q, k, v, o, lse, ent)
        ctx.sm_scale = sm_scale
        ctx.set_materialize_grads(False)
        return o, ent

    @staticmethod
    def backward(ctx, do, de):
        q, k, v, o, lse, ent = ctx.saved_tensors
        if do is None:
            do = torch.zeros_like(o)
        do = do.to(q.dtype)
        do = do if (q.size(-1), do.size(-1)) in ((128, 128), (64, 64)) and ops.viewable(do) else do.contiguous()
        if de is not None:
            de = de.float().contiguous()
        # empty_like keeps a dense or token-major input's strides for its gradient
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ops.fea_bwd(q, k, v, o, do, lse, dq, dk, dv, ctx.sm_scale, ent=ent, dent=de, grad_mode=0)
        return dq, dk, dv, None, None


def flash_entropy_attention(q, k, v, sm_scale=None, warp_specialize=True):
    """
    Non-causal attention that also returns the entropy of every attention row.

    Args:
        q, k: (B, H, N, D)
        v: (B, H, N, Dv), Dv must be a multiple of D
        sm_scale: softmax scale, defaults to 1 / sqrt(D)
        warp_specialize: accepted for compatibility with the reference; ignored
    Returns:
        o: (B, H, N, Dv) = softmax(sm_scale * q k^T) v
        e: (B, H, N) float32, e_i = -sum_j P_ij log P_ij
    """
    _check_inputs(q, k, v)
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    return _FlashEntropyAttention.apply(q, k, v, sm_scale, warp_specialize)
