"""VMonarch attention in fp32 on the CPU (oracle; test infrastructure only).

Restates video_monarch_attention/vmonarch.py:29-69 with the R step (`_row_block_attention`,
vmonarch.py:19-26) replaced by dense fp32 entropy attention, exactly as the reference test
patches it (tests/test_vmonarch.py:55-59). Everything runs in fp32, so the casts of the reference's
bf16 path (`.to(q.dtype)`, vmonarch.py:59, 62-63) are identities here, as they are in the
reference's own fp32 oracle run (tests/test_vmonarch.py:60-62).

The L step is written column-major (one batched m x m problem per grid column j) with plain
matmuls rather than the reference's einsums, so the golden-vector comparison against the
reference (tests/golden/make_golden.py) is an independent check of the index bookkeeping.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .fea import entropy_attention


def r_step(u, kg, w):
    """R step (vmonarch.py:19-26): attention inside every grid row, sm_scale = 1.
    u, kg: (B, H, m, b, D); w: (B, H, m, b, Dw). Returns (out, ent) with ent NOT detached here;
    the caller detaches it as the reference does (vmonarch.py:26)."""
    out, ent = entropy_attention(u, kg, w, 1.0)
    return out, ent


def lstep_forward(qg, kr, ent, y=None, min_col_mass=0.01, scale=1.0):
    """One L step (vmonarch.py:53-63) for all grid columns at once.

    qg, kr: (B, H, m, b, D) grid-shaped queries and R-step keys; ent: (B, H, m, b) R-step row
    entropy (the reference's -neg_ent). With `y` (B, H, m, b, Dv) returns z (last iteration,
    vmonarch.py:57-59); otherwise returns (u, col_mass) (vmonarch.py:61-63)."""
    qc = qg.transpose(2, 3)                          # (B, H, b, m, D): column j, rows i
    kc = kr.transpose(2, 3)                          # (B, H, b, m, D): column j, rows k
    bias = ent.transpose(2, 3).unsqueeze(-2)         # (B, H, b, 1, m): ent[k, j]
    a = torch.softmax(qc @ kc.transpose(-1, -2) + bias, dim=-1)   # (B, H, b, m_i, m_k)
    if y is not None:
        return (a @ y.transpose(2, 3)).transpose(2, 3)            # z[i, j] = sum_k a_ik y[k, j]
    col_mass = a.sum(-2).clamp_min(min_col_mass)                  # (B, H, b, m_k)
    uc = (a.transpose(-1, -2) @ qc) * (scale / col_mass).unsqueeze(-1)
    return uc.transpose(2, 3), col_mass.transpose(2, 3)


def vmonarch_attention(q, k, v, num_blocks, block_size, num_iters=2, recompute_tokens=0, min_col_mass=0.01):
    """fp32 VMonarch forward; differentiable through torch autograd (vmonarch.py:29-69)."""
    q, k, v = q.float(), k.float(), v.float()
    B, H, N, D = q.shape
    assert N == num_blocks * block_size, f"N={N} != {num_blocks} * {block_size}"
    if num_iters < 1:
        raise UnboundLocalError("cannot access local variable 'z' where it is not associated with a value")
    scale = D ** -0.5
    grid = (num_blocks, block_size)
    qg, kg, vg = q.unflatten(2, grid), k.unflatten(2, grid), v.unflatten(2, grid)
    u = qg * scale                                                   # vmonarch.py:47
    for it in range(num_iters):
        if it == num_iters - 1:
            out, ent = r_step(u, kg, torch.cat([kg, vg], dim=-1))    # vmonarch.py:50
            z = lstep_forward(qg, out[..., :D] * scale, ent.detach(), y=out[..., D:])
        else:
            out, ent = r_step(u, kg, kg)
            u, _ = lstep_forward(qg, out * scale, ent.detach(), min_col_mass=min_col_mass, scale=scale)
    z = z.reshape(B, H, N, -1)                                       # vmonarch.py:65
    r = recompute_tokens
    if r > 0:                                                        # vmonarch.py:66-68
        exact = F.scaled_dot_product_attention(q[:, :, :r], k, v)
        z = torch.cat([exact, z[:, :, r:]], dim=2)
    return z
