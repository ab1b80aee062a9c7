"""Entropy attention in fp32 on the CPU (oracle; test infrastructure only).

Restates the reference's dense check ``entropy_attention_ref`` (tests/test_vmonarch.py:12-15):
    logp = log_softmax(sm_scale q k^T);  o = exp(logp) v;  e = -sum exp(logp) logp
which is the function the Triton kernel computes (video_monarch_attention/kernel.py:32-151):
o = softmax(s) v (kernel.py:148) and e = log l - h / l (kernel.py:146) = -sum p log p.
"""
from __future__ import annotations

import torch


def entropy_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float):
    """o = softmax(sm_scale q k^T) v and e = row entropy, all in fp32 (differentiable)."""
    logp = (sm_scale * q.float() @ k.float().transpose(-1, -2)).log_softmax(-1)
    p = logp.exp()
    return p @ v.float(), -(p * logp).sum(-1)


def entropy_attention_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float,
                           rows: torch.Tensor):
    """The same for a subset of query rows (index tensor over dim -2): used to check full-size
    GPU outputs on sampled rows, since every row of attention is independent of the others."""
    return entropy_attention(q.index_select(-2, rows), k, v, sm_scale)
