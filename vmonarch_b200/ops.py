"""Thin tensor-level wrappers around the C-ABI entry points (one function per entry point).

All tensors must be CUDA tensors on the same device, with contiguous rows; batch strides are
taken from the tensors. Work is enqueued on the current torch stream of that device.
"""
from __future__ import annotations

import ctypes
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


def _bs(t: torch.Tensor, rows_dims: int = 2) -> int:
    """Batch stride (elements) of a tensor viewed as [batch][rows][cols] with contiguous rows."""
    if t.stride(-1) != 1 or (t.dim() >= 2 and t.size(-2) > 1 and t.stride(-2) != t.size(-1)):
        raise AssertionError("rows must be contiguous")
    return t.stride(-3) if t.dim() >= 3 else t.size(-2) * t.size(-1)


def _flat3(t: torch.Tensor) -> torch.Tensor:
    """View [..., rows, cols] as [batch, rows, cols] without copying (batch dims must be uniform).

    ``view`` (not ``reshape``) so that an output can never silently become a copy."""
    if t.dim() == 3:
        return t
    return t.view(-1, t.size(-2), t.size(-1))


def fea_fwd(q, k, v, o, lse, ent, sm_scale: float, v2=None) -> None:
    """o[b] = softmax(sm_scale q[b] k[b]^T) [v[b] | v2[b]]; lse/ent per query row (see header)."""
    q3, k3, v3, o3 = _flat3(q), _flat3(k), _flat3(v), _flat3(o)
    v23 = _flat3(v2) if v2 is not None else None
    a = N.FeaFwdArgs()
    a.q, a.q_bs = q3.data_ptr(), _bs(q3)
    a.k, a.k_bs = k3.data_ptr(), _bs(k3)
    a.v, a.v_bs = v3.data_ptr(), _bs(v3)
    if v23 is not None:
        a.v2, a.v2_bs = v23.data_ptr(), _bs(v23)
    a.o, a.o_bs = o3.data_ptr(), _bs(o3)
    a.lse = N.ptr(lse)
    a.ent = N.ptr(ent)
    a.batch, a.n_q, a.n_kv = q3.size(0), q3.size(1), k3.size(1)
    a.d, a.dv, a.dv1 = q3.size(2), o3.size(2), v3.size(2)
    a.dtype = N.dtype_code(q.dtype)
    a.sm_scale = float(sm_scale)
    nbytes = N.lib.vmb_fea_fwd_workspace_bytes(ctypes.byref(a))
    ws = None
    if nbytes > 0:  # lets the kernel split long key ranges over more CTAs
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    _call("vmb_fea_fwd", N.lib.vmb_fea_fwd, a, q.device)


def fea_bwd(q, k, v, o, dout, lse, grad_q, grad_k, grad_v, sm_scale: float, *, ent=None, dent=None, v2=None,
            grad_v2=None, grad_mode: int = 0, v_is_k: bool = False, delta=None, deterministic=None, fin_q=None,
            fin_k=None, fin_v=None, fin_v2=None) -> None:
    """Backward of :func:`fea_fwd`; see ``vmb_fea_bwd`` in the header for the modes. ``deterministic``
    (default: ``torch.are_deterministic_algorithms_enabled()``) rules out concurrent fp32 reductions;
    ``fin_*`` are the fp32 accumulators of grad_mode 3 (16-bit grad_* = fin_* + this gradient)."""
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled()
    q3, k3, v3, o3, do3 = _flat3(q), _flat3(k), _flat3(v), _flat3(o), _flat3(dout)
    a = N.FeaBwdArgs()
    a.q, a.q_bs = q3.data_ptr(), _bs(q3)
    a.k, a.k_bs = k3.data_ptr(), _bs(k3)
    a.v, a.v_bs = v3.data_ptr(), _bs(v3)
    if v2 is not None:
        v23 = _flat3(v2)
        a.v2, a.v2_bs = v23.data_ptr(), _bs(v23)
    a.o, a.o_bs = o3.data_ptr(), _bs(o3)
    a.dout, a.do_bs = do3.data_ptr(), _bs(do3)
    a.lse, a.ent, a.dent = N.ptr(lse), N.ptr(ent), N.ptr(dent)
    a.delta = N.ptr(delta)  # optional sum o . dout per query row (e.g. from lstep_bwd's delta_out)
    gq3, gk3 = _flat3(grad_q), _flat3(grad_k)
    a.grad_q, a.grad_q_bs = gq3.data_ptr(), _bs(gq3)
    a.grad_k, a.grad_k_bs = gk3.data_ptr(), _bs(gk3)
    if grad_v is not None:
        gv3 = _flat3(grad_v)
        a.grad_v, a.grad_v_bs = gv3.data_ptr(), _bs(gv3)
    if grad_v2 is not None:
        gv23 = _flat3(grad_v2)
        a.grad_v2, a.grad_v2_bs = gv23.data_ptr(), _bs(gv23)
    a.batch, a.n_q, a.n_kv = q3.size(0), q3.size(1), k3.size(1)
    a.d, a.dv, a.dv1 = q3.size(2), o3.size(2), v3.size(2)
    a.dtype = N.dtype_code(q.dtype)
    a.grad_mode = grad_mode
    a.v_is_k = int(v_is_k)
    a.sm_scale = float(sm_scale)
    a.deterministic = int(bool(deterministic))
    for name, t in (("fin_q", fin_q), ("fin_k", fin_k), ("fin_v", fin_v), ("fin_v2", fin_v2)):
        if t is not None:
            t3 = _flat3(t)
            setattr(a, name, t3.data_ptr())
            setattr(a, name + "_bs", _bs(t3))
    chunk, nbytes = bwd_plan(a)
    try:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    except torch.OutOfMemoryError:
        # no room for the preferred workspace: one call with the minimal one
        chunk, nbytes = a.batch, N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a))
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    if chunk >= a.batch:
        _call("vmb_fea_bwd", N.lib.vmb_fea_bwd, a, q.device)
        return
    for start in range(0, a.batch, chunk):
        _call("vmb_fea_bwd", N.lib.vmb_fea_bwd, _bwd_chunk(a, start, min(chunk, a.batch - start)), q.device)


def set_workspace_limit(nbytes: int) -> None:
    """Sets the upper bound (bytes) of one backward call's workspace (see ``bwd_plan``)."""
    global _workspace_limit
    _workspace_limit = int(nbytes)


def workspace_limit() -> int:
    return _workspace_limit


def bwd_plan(a: N.FeaBwdArgs) -> tuple[int, int]:
    """(sequences per call, workspace bytes) of a backward call under the workspace bound: the whole
    batch with its preferred workspace when that fits; else the fewest equal batch chunks whose
    preferred workspace fits and still holds the dS^T buffer; else the whole batch with the minimal
    workspace."""
    pref = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(a))
    low = N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(a))
    batch = a.batch
    if pref <= _workspace_limit or pref <= low or batch <= 1:
        return batch, pref
    b = _copy_args(a)
    c = max(2, -(-pref // max(_workspace_limit, 1)))
    while c <= batch:
        b.batch = -(-batch // c)
        p = N.lib.vmb_fea_bwd_workspace_bytes(ctypes.byref(b))
        if p <= _workspace_limit:
            if p > N.lib.vmb_fea_bwd_min_workspace_bytes(ctypes.byref(b)):
                return b.batch, p
            break  # chunks this small no longer take the dS^T route
        c += 1
    return batch, low


def _copy_args(a):
    b = type(a)()
    ctypes.memmove(ctypes.byref(b), ctypes.byref(a), ctypes.sizeof(a))
    return b


def _bwd_chunk(a: N.FeaBwdArgs, start: int, count: int) -> N.FeaBwdArgs:
    """The arguments of sequences [start, start + count) of a backward call (same workspace)."""
    b = _copy_args(a)
    b.batch = count
    g = 4 if a.grad_mode in (1, 2) else 2  # element size of the gradients

    def off(name, stride_elems, elem):
        base = getattr(a, name)
        if base:
            setattr(b, name, base + start * stride_elems * elem)

    for name, bs in (("q", "q_bs"), ("k", "k_bs"), ("v", "v_bs"), ("v2", "v2_bs"), ("o", "o_bs"), ("dout", "do_bs")):
        off(name, getattr(a, bs), 2)
    for name in ("lse", "ent", "dent", "delta"):
        off(name, a.n_q, 4)
    for name in ("grad_q", "grad_k", "grad_v", "grad_v2"):
        off(name, getattr(a, name + "_bs"), g)
    for name in ("fin_q", "fin_k", "fin_v", "fin_v2"):
        off(name, getattr(a, name + "_bs"), 4)
    return b


def _lstep_args(q, out, ent, m: int, b: int, scale: float, min_col_mass: float, last: bool, skip_rows: int):
    a = N.LstepArgs()
    a.q, a.out, a.ent = q.data_ptr(), out.data_ptr(), ent.data_ptr()
    a.bh = q.numel() // (m * b * q.size(-1))
    a.m, a.b = m, b
    a.d, a.dw = q.size(-1), out.size(-1)
    a.dtype = N.dtype_code(q.dtype)
    a.last = int(last)
    a.skip_rows = skip_rows
    a.scale, a.min_col_mass = float(scale), float(min_col_mass)
    return a


def lstep_fwd(q, out, ent, m: int, b: int, scale: float, min_col_mass: float, *, u=None, z=None,
              skip_rows: int = 0) -> None:
    """Monarch L step forward: writes u (non-last) or z (last, tokens >= skip_rows)."""
    a = _lstep_args(q, out, ent, m, b, scale, min_col_mass, z is not None, skip_rows)
    a.u, a.z = N.ptr(u), N.ptr(z)
    _call("vmb_lstep_fwd", N.lib.vmb_lstep_fwd, a, q.device)


def lstep_bwd(q, out, ent, m: int, b: int, scale: float, min_col_mass: float, dq, dout, *, du=None, dz=None,
              skip_rows: int = 0, dq_store: bool = False, delta_out=None) -> None:
    """Monarch L step backward: adds into dq (fp32; overwrites it when dq_store), writes dout (gradient
    of the R-step output) and, when given, delta_out = sum out . dout per token (fp32)."""
    a = _lstep_args(q, out, ent, m, b, scale, min_col_mass, dz is not None, skip_rows)
    a.du, a.dz, a.dq, a.dout = N.ptr(du), N.ptr(dz), dq.data_ptr(), dout.data_ptr()
    a.dq_store = int(dq_store)
    a.delta_out = N.ptr(delta_out)
    _call("vmb_lstep_bwd", N.lib.vmb_lstep_bwd, a, q.device)


def cast_f32(src: torch.Tensor, dst: torch.Tensor) -> None:
    """dst = src (fp32 -> dst.dtype). Both [batch][rows][cols] views with contiguous rows and the same
    shape (e.g. the same row range of two per-head tensors)."""
    s3, d3 = _flat3(src), _flat3(dst)
    assert s3.shape == d3.shape
    n = s3.size(1) * s3.size(2)
    if n == 0 or s3.size(0) == 0:
        return
    N.check(N.lib.vmb_cast_f32(s3.data_ptr(), _bs(s3), d3.data_ptr(), _bs(d3), s3.size(0), n, N.dtype_code(dst.dtype),
                               N.stream_ptr(src.device)), "vmb_cast_f32")
