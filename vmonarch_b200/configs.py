"""Seeded synthetic workloads standing in for the reference's video-DiT attention layers.

The reference publishes no dataset or benchmark inputs; these are the five configurations the
benchmark is quoted on, with the shapes and value distributions they describe:
  cpu_plumbing  B=1 H=2  m=4  b=64   D=64   iters=2 r=64     q,k,v ~ N(0,1)
  readme        B=2 H=4  m=16 b=256  D=128  iters=2 r=256    q,k,v ~ N(0,1)    (README usage shape)
  fea32k        B=1 H=24 N=32768     D=128  FEA fwd+bwd      q,k ~ N(0,1) + per-1024-token-block
                                                             shared N(0, 0.5^2) vector; v ~ N(0,1);
                                                             dO ~ N(0,1), dE ~ N(0, 0.1^2)
  dit14b        B=1 H=40 m=21 b=1560 D=128  iters=2 r=1560   q,k,v ~ N(0,1) + per-frame shared
                                                             N(0, 0.3^2) mean
  long720p      B=1 H=40 m=32 b=3600 D=128  iters=3 r=3600   same distribution as dit14b
Values are generated per (batch, head) from a generator seeded by (seed, batch, head), so any
head slice (multi-GPU sharding, CPU baseline samples) reproduces exactly the same numbers.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    H: int
    D: int
    Dv: int
    m: int = 1            # num_blocks (VMonarch) ; 1 for the plain FEA workload
    b: int = 0            # block_size (VMonarch) ; N for the plain FEA workload
    iters: int = 2
    recompute: int = 0
    kind: str = "vmonarch"          # "vmonarch" | "fea"
    shared: str = "none"            # "none" | "frame" | "block1024"
    shared_std: float = 0.0

    @property
    def N(self) -> int:
        return self.m * self.b

    def flops(self) -> dict:
        """Algorithmic FLOPs (unpadded; 2 per multiply-add) of one forward and one backward."""
        B, H, N, D, Dv = self.B, self.H, self.N, self.D, self.Dv
        if self.kind == "fea":
            fwd = 2.0 * B * H * N * N * (D + Dv)
            return {"fwd": fwd, "bwd": 2.5 * fwd, "dense_fwd": fwd}
        m, b, r = self.m, self.b, min(self.recompute, N)
        S = B * H * m
        fwd = bwd = 0.0
        for it in range(self.iters):
            Dw = D + Dv if it == self.iters - 1 else D
            fwd += 2.0 * S * b * b * (D + Dw)                  # R step
            bwd += 2.0 * S * b * b * (3 * D + 2 * Dw)
            lf = 2.0 * B * H * b * m * m * (D + (Dv if it == self.iters - 1 else D))
            fwd += lf                                          # L step
            bwd += 2.0 * lf
        fwd += 2.0 * B * H * r * N * (D + Dv)                  # exact recompute
        bwd += 2.0 * B * H * r * N * (3 * D + 2 * Dv)
        return {"fwd": fwd, "bwd": bwd, "dense_fwd": 2.0 * B * H * N * N * (D + Dv)}


WORKLOADS = {
    "cpu_plumbing": Workload("cpu_plumbing", B=1, H=2, D=64, Dv=64, m=4, b=64, iters=2, recompute=64),
    "readme": Workload("readme", B=2, H=4, D=128, Dv=128, m=16, b=256, iters=2, recompute=256),
    "fea32k": Workload("fea32k", B=1, H=24, D=128, Dv=128, m=1, b=32768, kind="fea", shared="block1024",
                       shared_std=0.5),
    "dit14b": Workload("dit14b", B=1, H=40, D=128, Dv=128, m=21, b=1560, iters=2, recompute=1560, shared="frame",
                       shared_std=0.3),
    "long720p": Workload("long720p", B=1, H=40, D=128, Dv=128, m=32, b=3600, iters=3, recompute=3600,
                         shared="frame", shared_std=0.3),
}


def _gen(seed: int, bi: int, h: int, salt: int) -> torch.Generator:
    return torch.Generator().manual_seed(((seed * 1000003 + bi) * 1009 + h) * 17 + salt)


def make_head(w: Workload, seed: int, bi: int, h: int):
    """fp32 CPU q, k, v, dO, dE for one (batch, head): (N, D), (N, D), (N, Dv), (N, Dv), (N,)."""
    N, D, Dv = w.N, w.D, w.Dv
    g = _gen(seed, bi, h, 0)
    q = torch.randn(N, D, generator=g)
    k = torch.randn(N, D, generator=g)
    v = torch.randn(N, Dv, generator=g)
    if w.shared == "block1024":
        nb = (N + 1023) // 1024
        c = torch.randn(nb, D, generator=g) * w.shared_std
        cb = c.repeat_interleave(1024, dim=0)[:N]
        q += cb
        k += cb
    elif w.shared == "frame":
        mu_q = torch.randn(w.m, D, generator=g) * w.shared_std
        mu_k = torch.randn(w.m, D, generator=g) * w.shared_std
        mu_v = torch.randn(w.m, Dv, generator=g) * w.shared_std
        q += mu_q.repeat_interleave(w.b, dim=0)
        k += mu_k.repeat_interleave(w.b, dim=0)
        v += mu_v.repeat_interleave(w.b, dim=0)
    g2 = _gen(seed, bi, h, 1)
    do = torch.randn(N, Dv, generator=g2)
    de = torch.randn(N, generator=g2) * 0.1
    return q, k, v, do, de


def make_inputs(w: Workload, seed: int = 0, heads: range | None = None, dtype=torch.bfloat16, device="cpu",
                pin: bool = False):
    """Stacked (B, Hs, N, ·) q, k, v, dO and (B, Hs, N) dE for the heads in `heads` (default all),
    rounded to `dtype` (dE stays fp32)."""
    heads = range(w.H) if heads is None else heads
    per = [[make_head(w, seed, bi, h) for h in heads] for bi in range(w.B)]

    def stack(i, dt):
        t = torch.stack([torch.stack([p[i] for p in row]) for row in per]).to(dt)
        if pin:
            t = t.pin_memory()
        return t.to(device) if device != "cpu" else t

    return stack(0, dtype), stack(1, dtype), stack(2, dtype), stack(3, dtype), stack(4, torch.float32)
