"""
VMonarch attention on the B200 kernels.

Drop-in for ``video_monarch_attention.vmonarch`` (reference ``video_monarch_attention/vmonarch.py``).
The N = m * b tokens lie on an (m, b) grid, token n -> (n // b, n % b). The attention map is
approximated by a Monarch matrix: R = m dense (b x b) blocks mixing tokens inside a grid row, and
L = b dense (m x m) blocks mixing tokens inside a grid column, fitted by `num_iters` steps of
alternating minimisation (reference vmonarch.py:1-11).

Layouts: q, k, v may be dense (B, H, N, D) or token-major, i.e. (B, N, H, D) buffers seen through
transpose(1, 2) as the Video-DiT caller holds them (reference README.md:74-76); the kernels read and
write them in place through strided layouts, and z and the gradients come back in the same layout
family (no transposes on either side).

Execution per iteration (all on the C ABI, no torch math on the hot path):
  R step: FlashEntropyAttention over the B*H*m grid rows (vmb_fea_fwd, entropy on). The first
          iteration folds the reference's u = q * scale (vmonarch.py:47) into sm_scale, and the last
          iteration reads [k | v] through two value pointers instead of torch.cat (vmonarch.py:50).
  L step: one fused kernel per iteration (vmb_lstep_fwd) for the einsum / softmax / column mass /
          rescale of vmonarch.py:51-63.
Recompute: the first `recompute_tokens` queries run exact attention (vmb_fea_fwd without entropy)
          written straight into rows [0, r) of z, replacing SDPA + torch.cat (vmonarch.py:66-68).
FP8 R step (opt-in, `fp8_r_step=True`; no reference counterpart): q, k, v and each iteration's u
          are rounded to e4m3 (vmb_quant_e4m3, saturating at +-448) and the R steps' two products run
          on the fp8 tensor cores with P in e4m3 too; the L steps, the recompute and the whole
          backward stay 16-bit (the backward differentiates the 16-bit R step at the same inputs).
The backward is hand-derived (the reference relies on autograd through the same ops) and
accumulates dq / dk / dv in fp32 across the recompute and every R and L step.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops
from .kernel import _check_inputs


def _token_major(t: torch.Tensor) -> bool:
    """(B, H, N, D) tensor whose tokens are further apart than its heads: a (B, N, H, D) buffer
    seen through transpose(1, 2), the Video-DiT layout (reference README.md:74-76)."""
    return t.size(1) > 1 and t.size(2) > 1 and t.stride(1) < t.stride(2)


def _alloc_like_layout(ref: torch.Tensor, cols: int, dtype) -> torch.Tensor:
    """(B, H, N, cols) output in `ref`'s layout family: token-major when `ref` is, else dense."""
    B, H, N, _ = ref.shape
    if _token_major(ref):
        return torch.empty((B, N, H, cols), device=ref.device, dtype=dtype).transpose(1, 2)
    return torch.empty((B, H, N, cols), device=ref.device, dtype=dtype)


def _in_place(t: torch.Tensor, strided: bool) -> torch.Tensor:
    """`t` itself when the kernels can read it through its strides (dense or token-major; the D = 128
    kernels with m <= 128 take any such layout), else a dense copy."""
    return t if strided and ops.viewable(t) else t.contiguous()


class _VMonarchAttention(torch.autograd.Function):
    """Tensors keep the caller's layout: q, k, v, z and the gradients are (B, H, N, .) views, dense
    or token-major, read and written in place through strided layouts; the R-step outputs, the next
    queries u and the fp32 gradient accumulators are dense internal buffers."""

    @staticmethod
    def forward(ctx, q, k, v, num_blocks, block_size, num_iters, recompute_tokens, min_col_mass, fp8_r_step=False):
        B, H, N, D = q.shape
        Dv = v.shape[-1]
        m, b = num_blocks, block_size
        scale = D ** -0.5
        strided = D == 128 and Dv == 128 and m <= 128
        qs, ks, vs = (_in_place(t, strided) for t in (q, k, v))
        dev, dt = q.device, q.dtype
        rr = min(max(int(recompute_tokens), 0), N)
        grid = lambda t: t.unflatten(2, (m, b))  # noqa: E731  (B, H, m, b, .): grid rows as FEA batches

        steps = []
        u = qs
        z = None
        if fp8_r_step:  # e4m3 operands of the R steps (dense copies; u is rounded per iteration)
            k8, v8 = ops.quant_e4m3(ks), ops.quant_e4m3(vs)
        for it in range(num_iters):
            last = it == num_iters - 1
            Dw = D + Dv if last else D
            out = torch.empty((B, H, N, Dw), device=dev, dtype=dt)
            lse = torch.empty((B, H, N), device=dev, dtype=torch.float32)
            ent = torch.empty((B, H, N), device=dev, dtype=torch.float32)
            sm = scale if it == 0 else 1.0
            if fp8_r_step:
                ops.fea_fwd(grid(ops.quant_e4m3(u)), grid(k8), grid(k8), grid(out), lse, ent, sm,
                            v2=grid(v8) if last else None)
            else:
                ops.fea_fwd(grid(u), grid(ks), grid(ks), grid(out), lse, ent, sm, v2=grid(vs) if last else None)
            if last:
                z = _alloc_like_layout(qs, Dv, dt)
                # every token of z is produced here (the tensor-core L step writes whole stacked
                # columns); the exact recompute below then overwrites tokens [0, rr)
                ops.lstep_fwd(qs, out, ent, m, b, scale, min_col_mass, z=z, skip_rows=0)
                nxt = None
            else:
                nxt = torch.empty((B, H, N, D), device=dev, dtype=dt)
                ops.lstep_fwd(qs, out, ent, m, b, scale, min_col_mass, u=nxt)
            steps.append((u, out, lse, ent, sm))
            u = nxt

        lse_r = None
        if rr > 0:
            lse_r = torch.empty((B, H, rr), device=dev, dtype=torch.float32)
            ops.fea_fwd(qs[:, :, :rr], ks, vs, z[:, :, :rr], lse_r, None, scale)

        ctx.meta = (B, H, N, D, Dv, m, b, rr, scale, min_col_mass, strided)
        if any(ctx.needs_input_grad[:3]):
            flat = [qs, ks, vs, z] + ([lse_r] if lse_r is not None else [])
            for st in steps:
                flat.extend(st[:4])
            ctx.save_for_backward(*flat)
            ctx.sms = [st[4] for st in steps]
        return z

    @staticmethod
    def backward(ctx, dz):
        B, H, N, D, Dv, m, b, rr, scale, min_col_mass, strided = ctx.meta
        saved = ctx.saved_tensors
        qs, ks, vs, z = saved[:4]
        pos = 4
        lse_r = None
        if rr > 0:
            lse_r = saved[4]
            pos = 5
        steps = [saved[pos + 4 * i: pos + 4 * i + 4] for i in range(len(ctx.sms))]
        dev, dt = qs.device, qs.dtype
        dz = _in_place(dz.to(dt), strided)
        grid = lambda t: t.unflatten(2, (m, b))  # noqa: E731

        # fp32 accumulators. Each is first written by a call that covers all of its rows and
        # OVERWRITES it (no zero-fill): dq by the last L step, dk / dv (and every R step's own dq,
        # gq) by the last R step; later calls add. The recompute's contribution comes last.
        dq_acc = torch.empty((B, H, N, D), device=dev, dtype=torch.float32)
        dk_acc = torch.empty((B, H, N, D), device=dev, dtype=torch.float32)
        dv_acc = torch.empty((B, H, N, Dv), device=dev, dtype=torch.float32)
        kv_fresh = True   # dk_acc / dv_acc not yet written

        du = None
        n_it = len(steps)
        for it in reversed(range(n_it)):
            u, out, lse, ent = steps[it]
            sm = ctx.sms[it]
            last = it == n_it - 1
            dout = torch.empty_like(out)
            # the L step also produces the R-step backward's delta = sum out . dout per token, so
            # the attention backward skips its own pass over out and dout
            delta = torch.empty((B, H, N), device=dev, dtype=torch.float32)
            if last:
                ops.lstep_bwd(qs, out, ent, m, b, scale, min_col_mass, dq_acc, dout, dz=dz, skip_rows=rr,
                              dq_store=True, delta_out=delta)
            else:
                ops.lstep_bwd(qs, out, ent, m, b, scale, min_col_mass, dq_acc, dout, du=du, delta_out=delta)
            gq = dq_acc if it == 0 else torch.empty((B, H, N, D), device=dev, dtype=torch.float32)
            gq_fresh = it != 0
            # one grad mode per call: overwrite only when every target is fresh, otherwise clear
            # the fresh ones and add (only with num_iters != 2)
            if gq_fresh and kv_fresh:
                mode = 2
            else:
                if gq_fresh:
                    gq.zero_()
                if kv_fresh:
                    dk_acc.zero_()
                    dv_acc.zero_()
                mode = 1
            ops.fea_bwd(grid(u), grid(ks), grid(ks), grid(out), grid(dout), lse, grid(gq), grid(dk_acc), None, sm,
                        v2=grid(vs) if last else None, grad_v2=grid(dv_acc) if last else None, grad_mode=mode,
                        v_is_k=True, delta=delta)
            kv_fresh = False
            du = gq

        dq = _alloc_like_layout(qs, D, dt)
        dk = _alloc_like_layout(ks, D, dt)
        dv = _alloc_like_layout(vs, Dv, dt)
        if rr > 0:
            # the recompute is the last contribution to dk, dv (every key) and dq[:rr]: it writes them
            # in the element dtype as accumulator + its own gradient (grad_mode 3)
            ops.fea_bwd(qs[:, :, :rr], ks, vs, z[:, :, :rr], dz[:, :, :rr], lse_r, dq[:, :, :rr], dk, dv, scale,
                        grad_mode=3, fin_q=dq_acc[:, :, :rr], fin_k=dk_acc, fin_v=dv_acc)
            ops.cast_f32(dq_acc[:, :, rr:], dq[:, :, rr:])
        else:
            ops.cast_f32(dq_acc, dq)
            ops.cast_f32(dk_acc, dk)
            ops.cast_f32(dv_acc, dv)
        return dq, dk, dv, None, None, None, None, None, None


def vmonarch_attention(q, k, v, num_blocks, block_size, num_iters=2, recompute_tokens=0, min_col_mass=0.01,
                       fp8_r_step=False):
    """
    Args:
        q, k: (B, H, N, D); v: (B, H, N, Dv), with N == num_blocks * block_size.
        num_blocks: m, number of grid rows (keep it small).
        block_size: b, number of tokens per grid row.
        num_iters: alternating-minimization steps.
        recompute_tokens: the first `recompute_tokens` queries use exact attention.
        min_col_mass: lower bound of the column mass of L, for stability.
        fp8_r_step: (B200 extension, default off) R-step attention on e4m3 operands; D = Dv = 128.
    Returns:
        (B, H, N, Dv)
    """
    B, H, N, D = q.shape
    assert N == num_blocks * block_size, f"N={N} != {num_blocks} * {block_size}"
    if num_iters < 1:
        # the reference leaves z unbound when the loop does not run (vmonarch.py:48-65)
        raise UnboundLocalError("cannot access local variable 'z' where it is not associated with a value")
    _check_inputs(q, k, v)
    Dv = v.shape[-1]
    # the last R step attends over [k | v] (vmonarch.py:50): its value width D + Dv must be a
    # multiple of D and a width the reference kernel accepts (kernel.py:260, 324)
    assert (D + Dv) % D == 0 and D + Dv <= 256, f"D + Dv = {D + Dv} is not a valid last-step value width"
    # the L step keeps a grid column's m rows on chip: up to 128 on the tensor-core kernels (D in
    # {64, 128} with Dv == D), 64 on the generic kernel
    max_m = 128 if D in (64, 128) and Dv == D else 64
    if num_blocks > max_m:
        raise NotImplementedError(f"num_blocks={num_blocks} > {max_m}: the L step supports at most {max_m} grid rows "
                                  f"for D={D}, Dv={Dv}")
    if fp8_r_step and (D != 128 or Dv != 128):
        raise NotImplementedError(f"fp8_r_step needs D = Dv = 128 (got D={D}, Dv={Dv})")
    return _VMonarchAttention.apply(q, k, v, int(num_blocks), int(block_size), int(num_iters), recompute_tokens,
                                    float(min_col_mass), bool(fp8_r_step))


class VMonarchAttention(nn.Module):
    def __init__(self, num_blocks, block_size, num_iters=2, min_col_mass=0.01, fp8_r_step=False):
        super().__init__()
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_iters = num_iters
        self.min_col_mass = min_col_mass
        self.fp8_r_step = fp8_r_step

    def forward(self, q, k, v, recompute_tokens=0):
        return vmonarch_attention(q, k, v, self.num_blocks, self.block_size, self.num_iters,
                                  recompute_tokens, self.min_col_mass, self.fp8_r_step)

    def extra_repr(self):
        return f"num_blocks={self.num_blocks}, block_size={self.block_size}, num_iters={self.num_iters}"
