"""Thin tensor-level wrappers around the C-ABI entry points (one function per entry point).

Every tensor is a CUDA tensor of shape (*batch, rows, cols) with contiguous columns; all tensors
of a call share the batch shape, which has one to three dimensions. The tensors' own strides are
handed to the kernels as a strided layout (``vmb_fea_layout`` / ``vmb_lstep_layout`` in
include/vmonarch_b200.h), so a token-major caller tensor, a (B, N, H, D) buffer seen as
(B, H, N, D) through ``transpose(1, 2)``, is read and written in place: with batch shape (B, H)
the innermost batch dimension H is the layout's n1 and B its n2; with (B, H, m) grid rows (the
VMonarch R step) m is n1, H is n2 and B the outermost. Statistics (lse, ent, dent, delta) are
dense fp32 [batch][rows]. Work is enqueued on the current torch stream of the tensors' device.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _native as N

# Upper bound (bytes) of the workspace one backward call allocates. A call's preferred workspace can
# hold a dS^T buffer (2 bytes per query x key: 4.5 GB for the last R step of the 14B-class layer,
# ~35 GB for the 720p-class one); above the bound the call is issued over chunks of its batch that
# each fit, reusing one workspace, or with the minimal workspace (the dQ kernel that recomputes S
# and dP) when no chunk size keeps the dS^T route. VMONARCH_B200_WORKSPACE_LIMIT overrides it.
_workspace_limit = int(os.environ.get("VMONARCH_B200_WORKSPACE_LIMIT", 16 << 30))

# Optional per-call timer: a callable (name, flops_or_None) -> context manager, installed by the
# benchmark to bracket each C-ABI call with CUDA events on the current stream.
_timer = None


def set_timer(timer) -> None:
    global _timer
    _timer = timer


def kernel_launches() -> int:
    """Kernels launched by the library so far (vmb_kernel_launches)."""
    return int(N.lib.vmb_kernel_launches())


def _call(name: str, fn, arg, dev) -> None:
    if _timer is None:
        N.check(fn(ctypes.byref(arg), N.stream_ptr(dev)), name)
        return
    with _timer(name, arg):
        N.check(fn(ctypes.byref(arg), N.stream_ptr(dev)), name)


# ----------------------------------------------------------------------------------------- layouts
def viewable(t: torch.Tensor) -> bool:
    """True when the kernels can read or write `t` (shape (..., rows, cols)) in place: contiguous
    columns, 16-byte aligned base, every other stride a non-negative multiple of 16 bytes and rows
    at least `cols` apart. Otherwise the caller passes ``t.contiguous()``."""
    if t.dim() < 3 or t.stride(-1) != 1 or t.data_ptr() % 16:
        return False
    align = 16 // t.element_size()
    for i in range(t.dim() - 1):
        if t.size(i) > 1 and (t.stride(i) < 0 or t.stride(i) % align):
            return False
    return t.size(-2) <= 1 or t.stride(-2) >= t.size(-1)


def _view(t: torch.Tensor, nb: int) -> N.View:
    """The vmb_view of a (*batch[nb], rows, cols) tensor: row stride, then the strides of the
    innermost, middle and outermost batch dimension (0 for absent or size-1 dimensions)."""
    if t.stride(-1) != 1 and t.size(-1) > 1:
        raise AssertionError("columns must be contiguous")
    rows, cols = t.size(-2), t.size(-1)
    rs = t.stride(-2) if rows > 1 else cols
    st = [t.stride(-3 - i) if t.size(-3 - i) > 1 else 0 for i in range(nb)] + [0] * (3 - nb)
    return N.View(rs, st[0], st[1], st[2])


def _split(batch_shape) -> tuple[int, int]:
    """(n1, n2) of a batch shape: the innermost dimension, then the next one (1 if absent)."""
    if not 1 <= len(batch_shape) <= 3:
        raise AssertionError(f"batch shape {tuple(batch_shape)} must have one to three dimensions")
    return int(batch_shape[-1]), int(batch_shape[-2]) if len(batch_shape) >= 2 else 1


def _stats(t, batch: int, rows: int):
    if t is None:
        return None
    if not t.is_contiguous() or t.numel() != batch * rows or t.dtype != torch.float32:
        raise AssertionError("statistics must be contiguous fp32 [batch][rows]")
    return t.data_ptr()


# ----------------------------------------------------------------------------------------- forward
def fea_fwd(q, k, v, o, lse, ent, sm_scale: float, v2=None) -> None:
    """o = softmax(sm_scale q k^T) [v | v2] per batch entry; lse/ent per query row (see header).
    q, k, v (and v2) may be float8_e4m3fn (from quant_e4m3) for the R-step forms, o 16-bit."""
    bshape = q.shape[:-2]
    nb = len(bshape)
    for t in (k, v, o, v2):
        if t is not None and t.shape[:-2] != bshape:
            raise AssertionError("q, k, v, v2 and o must share their batch shape")
    n1, n2 = _split(bshape)
    batch = math.prod(bshape)
    lay = N.FeaLayout()
    lay.n1, lay.n2 = n1, n2
    a = N.FeaFwdArgs()
    for name, t in (("q", q), ("k", k), ("v", v), ("v2", v2), ("o", o)):
        if t is not None:
            setattr(a, name, t.data_ptr())
            setattr(lay, name, _view(t, nb))
    a.layout = ctypes.pointer(lay)
    a.lse = _stats(lse, batch, q.size(-2))
    a.ent = _stats(ent, batch, q.size(-2))
    a.batch, a.n_q, a.n_kv = batch, q.size(-2), k.size(-2)
    a.d, a.dv, a.dv1 = q.size(-1), o.size(-1), v.size(-1)
    a.dtype = N.dtype_code(o.dtype)
    e4m3 = q.dtype == torch.float8_e4m3fn
    if any((t.dtype == torch.float8_e4m3fn) != e4m3 for t in (k, v, v2) if t is not None):
        raise AssertionError("q, k, v and v2 must all be 16-bit or all e4m3")
    a.qkv_e4m3 = int(e4m3)
    a.sm_scale = float(sm_scale)
    nbytes = N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a))
    ws = None
    if nbytes > 0:  # lets the kernel split long key ranges over more CTAs
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    _call("vmb_fea_fwd", N.lib.vmb_fea_fwd, a, q.device)


# ----------------------------------------------------------------------------------------- backward
_BWD_TENSORS = ("q", "k", "v", "v2", "o", "dout", "grad_q", "grad_k", "grad_v", "grad_v2", "fin_q", "fin_k", "fin_v",
                "fin_v2")
_BWD_STATS = ("lse", "ent", "dent", "delta")


def bwd_args(t: dict, sm_scale: float, grad_mode: int, v_is_k: bool, deterministic: bool):
    """vmb_fea_bwd_args (and the layout it points to) for the tensors in `t` (names of
    _BWD_TENSORS and _BWD_STATS, absent or None when unused)."""
    q, k, o, v = t["q"], t["k"], t["o"], t["v"]
    bshape = q.shape[:-2]
    nb = len(bshape)
    n1, n2 = _split(bshape)
    batch = math.prod(bshape)
    lay = N.FeaLayout()
    lay.n1, lay.n2 = n1, n2
    a = N.FeaBwdArgs()
    for name in _BWD_TENSORS:
        x = t.get(name)
        if x is None:
            continue
        if x.shape[:-2] != bshape:
            raise AssertionError(f"{name} does not share the batch shape {tuple(bshape)}")
        setattr(a, name, x.data_ptr())
        setattr(lay, name, _view(x, nb))
    a.layout = ctypes.pointer(lay)
    for name in _BWD_STATS:
        setattr(a, name, _stats(t.get(name), batch, q.size(-2)))
    a.batch, a.n_q, a.n_kv = batch, q.size(-2), k.size(-2)
    a.d, a.dv, a.dv1 = q.size(-1), o.size(-1), v.size(-1)
    a.dtype = N.dtype_code(q.dtype)
    a.grad_mode = grad_mode
    a.v_is_k = int(v_is_k)
    a.sm_scale = float(sm_scale)
    a.deterministic = int(bool(deterministic))
    return a, lay


def fea_bwd(q, k, v, o, dout, lse, grad_q, grad_k, grad_v, sm_scale: float, *, ent=None, dent=None, v2=None,
            grad_v2=None, grad_mode: int = 0, v_is_k: bool = False, delta=None, deterministic=None, fin_q=None,
            fin_k=None, fin_v=None, fin_v2=None) -> None:
    """Backward of :func:`fea_fwd`; see ``vmb_fea_bwd`` in the header for the modes. ``deterministic``
    (default: ``torch.are_deterministic_algorithms_enabled()``) rules out concurrent fp32 reductions;
    ``fin_*`` are the fp32 accumulators of grad_mode 3 (16-bit grad_* = fin_* + this gradient)."""
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled()
    t = dict(q=q, k=k, v=v, v2=v2, o=o, dout=dout, grad_q=grad_q, grad_k=grad_k, grad_v=grad_v, grad_v2=grad_v2,
             fin_q=fin_q, fin_k=fin_k, fin_v=fin_v, fin_v2=fin_v2, lse=lse, ent=ent, dent=dent, delta=delta)
    a, lay = bwd_args(t, sm_scale, grad_mode, v_is_k, deterministic)
    bshape = q.shape[:-2]
    cdim = 1 if len(bshape) >= 2 else 0          # batch dimension the chunks run along
    unit = math.prod(bshape[cdim + 1:])          # sequences per index of that dimension
    chunk, nbytes = bwd_plan(a, unit=unit, group=unit * bshape[cdim])
    try:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    except torch.OutOfMemoryError:
        # no room for the preferred workspace: one call with the minimal one
        chunk, nbytes = a.batch, N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a))
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    if chunk >= a.batch:
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
        _call("vmb_fea_bwd", N.lib.vmb_fea_bwd, a, q.device)
        return
    # chunks of `chunk // unit` indices along batch dimension cdim, for every index of the outer ones
    n_q = q.size(-2)
    per = chunk // unit
    for outer in _outer_indices(bshape[:cdim]):
        for i0 in range(0, bshape[cdim], per):
            idx = outer + (slice(i0, min(i0 + per, bshape[cdim])),)
            sub = {}
            for name, x in t.items():
                if x is None:
                    continue
                if name in _BWD_STATS:
                    x = x.view(*bshape, n_q)
                sub[name] = x[idx]
                if name in _BWD_STATS:
                    sub[name] = sub[name].reshape(-1)  # contiguous: only outer dims are fixed
            b, lay_b = bwd_args(sub, sm_scale, grad_mode, v_is_k, deterministic)
            b.workspace, b.workspace_bytes = ws.data_ptr(), nbytes
            _call("vmb_fea_bwd", N.lib.vmb_fea_bwd, b, q.device)


def _outer_indices(shape):
    if not shape:
        yield ()
        return
    for i in range(shape[0]):
        for rest in _outer_indices(shape[1:]):
            yield (i,) + rest


def set_workspace_limit(nbytes: int) -> None:
    """Sets the upper bound (bytes) of one backward call's workspace (see ``bwd_plan``)."""
    global _workspace_limit
    _workspace_limit = int(nbytes)


def workspace_limit() -> int:
    return _workspace_limit


def bwd_plan(a: N.FeaBwdArgs, unit: int = 1, group: int = 0) -> tuple[int, int]:
    """(sequences per call, workspace bytes) of a backward call under the workspace bound: the whole
    batch with its preferred workspace when that fits; else the largest chunk (a multiple of `unit`
    sequences, at most `group`, so chunks never cross a `group` boundary) whose preferred workspace
    fits and still holds the dS^T buffer; else the whole batch with the minimal workspace."""
    pref = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a))
    low = N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a))
    batch = a.batch
    group = group or batch
    if pref <= _workspace_limit or pref <= low or batch <= unit:
        return batch, pref
    b = type(a)()
    ctypes.memmove(ctypes.byref(b), ctypes.byref(a), ctypes.sizeof(a))
    b.layout = None  # workspace sizes do not depend on the layout
    per = max(1, group // unit)  # indices of the chunked dimension
    last = None
    for c in range(1, per + 1):
        k = -(-per // c)
        if k == last:
            continue
        last = k
        b.batch = k * unit
        if b.batch >= batch:
            continue  # not a split
        p = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(b))
        if p <= _workspace_limit:
            return (b.batch, p) if p > N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(b)) else (batch, low)
    return batch, low


# ----------------------------------------------------------------------------------------- L step
def _lstep_args(q, out, ent, m: int, b: int, scale: float, min_col_mass: float, last: bool, skip_rows: int,
                tensors: dict):
    """Arguments and layout of an L-step call. q, out and the tensors in `tensors` are (BH, N, C) or
    (B, H, N, C) with N = m * b tokens; ent (and delta_out) are dense fp32 [bh][N]."""
    bshape = q.shape[:-2]
    nb = len(bshape)
    if nb not in (1, 2):
        raise AssertionError("L-step tensors are (BH, N, C) or (B, H, N, C)")
    lay = N.LstepLayout()
    lay.n1 = int(bshape[-1])
    a = N.LstepArgs()
    for name, t in dict(q=q, out=out, **tensors).items():
        if t is None or name == "delta_out":
            continue
        if t.shape[:-2] != bshape or t.size(-2) != m * b:
            raise AssertionError(f"{name} must be {tuple(bshape)} x {m * b} tokens")
        setattr(a, name, t.data_ptr())
        v = _view(t, nb)
        setattr(lay, name, N.View(v.row, v.s1, 0, v.s2))  # L-step views: head hb at (hb % n1) s1 + (hb / n1) s3
    bh = math.prod(bshape)
    a.layout = ctypes.pointer(lay)
    a.ent = _stats(ent, bh, m * b)
    a.delta_out = _stats(tensors.get("delta_out"), bh, m * b)
    a.bh = bh
    a.m, a.b = m, b
    a.d, a.dw = q.size(-1), out.size(-1)
    a.dtype = N.dtype_code(q.dtype)
    a.last = int(last)
    a.skip_rows = skip_rows
    a.scale, a.min_col_mass = float(scale), float(min_col_mass)
    return a, lay


def lstep_fwd(q, out, ent, m: int, b: int, scale: float, min_col_mass: float, *, u=None, z=None,
              skip_rows: int = 0) -> None:
    """Monarch L step forward: writes u (non-last) or z (last, tokens >= skip_rows)."""
    a, lay = _lstep_args(q, out, ent, m, b, scale, min_col_mass, z is not None, skip_rows, dict(u=u, z=z))
    _call("vmb_lstep_fwd", N.lib.vmb_lstep_fwd, a, q.device)


def lstep_bwd(q, out, ent, m: int, b: int, scale: float, min_col_mass: float, dq, dout, *, du=None, dz=None,
              skip_rows: int = 0, dq_store: bool = False, delta_out=None) -> None:
    """Monarch L step backward: adds into dq (fp32; overwrites it when dq_store), writes dout (gradient
    of the R-step output) and, when given, delta_out = sum out . dout per token (fp32)."""
    a, lay = _lstep_args(q, out, ent, m, b, scale, min_col_mass, dz is not None, skip_rows,
                         dict(du=du, dz=dz, dq=dq, dout=dout, delta_out=delta_out))
    a.dq_store = int(dq_store)
    _call("vmb_lstep_bwd", N.lib.vmb_lstep_bwd, a, q.device)


def quant_e4m3(src: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """e4m3(scale * src) as a new dense float8_e4m3fn tensor of src's shape; src 16-bit, (*batch,
    rows, cols) with cols a multiple of 16, any strides the kernels can read in place (dense or
    token-major). Rounded to nearest, saturating at +-448."""
    bshape = src.shape[:-2]
    nb = len(bshape)
    dst = torch.empty(src.shape, dtype=torch.float8_e4m3fn, device=src.device)
    if src.numel() == 0:
        return dst
    src = src if viewable(src) else src.contiguous()
    n1, n2 = _split(bshape)
    sv, dv = _view(src, nb), _view(dst, nb)
    N.check(N.lib.vmb_quant_e4m3(src.data_ptr(), ctypes.byref(sv), dst.data_ptr(), ctypes.byref(dv), n1, n2,
                                 math.prod(bshape), src.size(-2), src.size(-1), N.dtype_code(src.dtype), float(scale),
                                 N.stream_ptr(src.device)), "vmb_quant_e4m3")
    return dst


def cast_f32(src: torch.Tensor, dst: torch.Tensor) -> None:
    """dst = src (fp32 -> dst.dtype), both (*batch, rows, cols) with the same shape, any strides the
    kernels can read in place (e.g. the same row range of an fp32 accumulator and of a token-major
    gradient)."""
    assert src.shape == dst.shape and src.dtype == torch.float32
    bshape = src.shape[:-2]
    nb = len(bshape)
    if src.numel() == 0:
        return
    n1, n2 = _split(bshape)
    sv, dv = _view(src, nb), _view(dst, nb)
    N.check(N.lib.vmb_cast_f32_view(src.data_ptr(), ctypes.byref(sv), dst.data_ptr(), ctypes.byref(dv), n1, n2,
                                    math.prod(bshape), src.size(-2), src.size(-1), N.dtype_code(dst.dtype),
                                    N.stream_ptr(src.device)), "vmb_cast_f32_view")
