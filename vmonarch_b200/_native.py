"""ctypes binding of the C ABI declared in ``include/vmonarch_b200.h``.

The library is the in-tree ``libvmonarch_b200.so`` built by :mod:`vmonarch_b200.build`. There is
no fallback: if the library is missing or fails to load, importing the package raises, and every
op raises if its inputs are not CUDA tensors.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("VMONARCH_B200_LIB", Path(__file__).resolve().parent / "libvmonarch_b200.so"))

VMB_DTYPE_BF16 = 0
VMB_DTYPE_F16 = 1
VMB_OK = 0
_ERRNAMES = {1: "EINVAL", 2: "ENOTSUP", 3: "ECUDA"}

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_vp = ctypes.c_void_p
c_fp = ctypes.POINTER(ctypes.c_float)


ABI_VERSION = 7  # VMB_ABI_VERSION of include/vmonarch_b200.h that these structures mirror


class View(ctypes.Structure):
    """vmb_view: element (s, r, c) at c + r*row + (s % n1)*s1 + (s / n1 % n2)*s2 + (s / (n1 n2))*s3."""
    _fields_ = [("row", c_i64), ("s1", c_i64), ("s2", c_i64), ("s3", c_i64)]


class FeaLayout(ctypes.Structure):
    _fields_ = [("n1", c_i64), ("n2", c_i64)] + [(n, View) for n in (
        "q", "k", "v", "v2", "o", "dout", "grad_q", "grad_k", "grad_v", "grad_v2", "fin_q", "fin_k", "fin_v",
        "fin_v2")]


class LstepLayout(ctypes.Structure):
    _fields_ = [("n1", c_i64)] + [(n, View) for n in ("q", "out", "u", "z", "du", "dz", "dq", "dout")]


class FeaFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_vp), ("q_bs", c_i64),
        ("k", c_vp), ("k_bs", c_i64),
        ("v", c_vp), ("v_bs", c_i64),
        ("v2", c_vp), ("v2_bs", c_i64),
        ("o", c_vp), ("o_bs", c_i64),
        ("lse", c_vp), ("ent", c_vp),
        ("batch", c_i64), ("n_q", c_i64), ("n_kv", c_i64),
        ("d", c_i32), ("dv", c_i32), ("dv1", c_i32), ("dtype", c_i32),
        ("sm_scale", ctypes.c_float),
        ("workspace", c_vp), ("workspace_bytes", c_i64),
        ("layout", ctypes.POINTER(FeaLayout)),
        ("qkv_e4m3", c_i32),
    ]


class FeaBwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_vp), ("q_bs", c_i64),
        ("k", c_vp), ("k_bs", c_i64),
        ("v", c_vp), ("v_bs", c_i64),
        ("v2", c_vp), ("v2_bs", c_i64),
        ("o", c_vp), ("o_bs", c_i64),
        ("dout", c_vp), ("do_bs", c_i64),
        ("lse", c_vp), ("ent", c_vp), ("dent", c_vp),
        ("grad_q", c_vp), ("grad_q_bs", c_i64),
        ("grad_k", c_vp), ("grad_k_bs", c_i64),
        ("grad_v", c_vp), ("grad_v_bs", c_i64),
        ("grad_v2", c_vp), ("grad_v2_bs", c_i64),
        ("workspace", c_vp), ("workspace_bytes", c_i64),
        ("batch", c_i64), ("n_q", c_i64), ("n_kv", c_i64),
        ("d", c_i32), ("dv", c_i32), ("dv1", c_i32), ("dtype", c_i32),
        ("grad_mode", c_i32), ("v_is_k", c_i32),
        ("sm_scale", ctypes.c_float),
        ("delta", c_vp),
        ("deterministic", c_i32),
        ("fin_q", c_vp), ("fin_q_bs", c_i64),
        ("fin_k", c_vp), ("fin_k_bs", c_i64),
        ("fin_v", c_vp), ("fin_v_bs", c_i64),
        ("fin_v2", c_vp), ("fin_v2_bs", c_i64),
        ("layout", ctypes.POINTER(FeaLayout)),
    ]


class LstepArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_vp), ("out", c_vp), ("ent", c_vp),
        ("u", c_vp), ("z", c_vp),
        ("du", c_vp), ("dz", c_vp),
        ("dq", c_vp), ("dout", c_vp),
        ("bh", c_i64), ("m", c_i64), ("b", c_i64),
        ("d", c_i32), ("dw", c_i32), ("dtype", c_i32), ("last", c_i32),
        ("skip_rows", c_i64),
        ("scale", ctypes.c_float), ("min_col_mass", ctypes.c_float),
        ("dq_store", c_i32),
        ("delta_out", c_vp),
        ("layout", ctypes.POINTER(LstepLayout)),
    ]


#: every symbol include/vmonarch_b200.h declares, with its ctypes signature
SIGNATURES = {
    "vmb_abi_version": (ctypes.c_int, []),
    "vmb_last_error": (ctypes.c_char_p, []),
    "vmb_kernel_launches": (ctypes.c_uint64, []),
    "vmb_test_pipeline_timeout": (ctypes.c_int, [c_i64, c_i32]),
    "vmb_device_status": (ctypes.c_int, [c_vp, ctypes.POINTER(ctypes.c_int32)]),
    "vmb_fea_fwd_workspace_bytes": (c_i64, [ctypes.POINTER(FeaFwdArgs)]),
    "vmb_fea_fwd": (ctypes.c_int, [ctypes.POINTER(FeaFwdArgs), c_vp]),
    "vmb_fea_bwd_workspace_bytes": (c_i64, [ctypes.POINTER(FeaBwdArgs)]),
    "vmb_fea_bwd_min_workspace_bytes": (c_i64, [ctypes.POINTER(FeaBwdArgs)]),
    "vmb_fea_bwd": (ctypes.c_int, [ctypes.POINTER(FeaBwdArgs), c_vp]),
    "vmb_fea_bwd_noalloc": (ctypes.c_int, [ctypes.POINTER(FeaBwdArgs), c_vp]),
    "vmb_lstep_fwd": (ctypes.c_int, [ctypes.POINTER(LstepArgs), c_vp]),
    "vmb_lstep_bwd": (ctypes.c_int, [ctypes.POINTER(LstepArgs), c_vp]),
    "vmb_cast_f32": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i32, c_vp]),
    "vmb_cast_f32_view": (ctypes.c_int, [c_vp, ctypes.POINTER(View), c_vp, ctypes.POINTER(View), c_i64, c_i64, c_i64,
                                         c_i64, c_i64, c_i32, c_vp]),
    "vmb_quant_e4m3": (ctypes.c_int, [c_vp, ctypes.POINTER(View), c_vp, ctypes.POINTER(View), c_i64, c_i64, c_i64,
                                      c_i64, c_i64, c_i32, ctypes.c_float, c_vp]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"vmonarch_b200: CUDA library {LIB_PATH} is missing; build it with `python vmonarch_b200/build.py`")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.vmb_abi_version.restype = ctypes.c_int
    if lib.vmb_abi_version() != ABI_VERSION:
        raise ImportError(f"vmonarch_b200: {LIB_PATH} has ABI version {lib.vmb_abi_version()}, the binding expects "
                          f"{ABI_VERSION}; rebuild it with `python vmonarch_b200/build.py`")
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class VMonarchError(RuntimeError):
    """Raised when a C-ABI call returns an error code."""


def check(rc: int, what: str) -> None:
    if rc != VMB_OK:
        msg = lib.vmb_last_error().decode(errors="replace")
        raise VMonarchError(f"{what} failed ({_ERRNAMES.get(rc, rc)}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return VMB_DTYPE_BF16
    if dt == torch.float16:
        return VMB_DTYPE_F16
    raise AssertionError(f"unsupported dtype {dt}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_status(device: torch.device) -> int:
    """OR of the pipeline-timeout codes recorded by the kernels since the last call (0 = none)."""
    out = ctypes.c_int32(0)
    check(lib.vmb_device_status(stream_ptr(device), ctypes.byref(out)), "vmb_device_status")
    return out.value


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
