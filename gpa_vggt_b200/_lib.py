"""ctypes binding of ``libgpa_b200.so`` (the C ABI in ``include/gpa_b200.h``).

The library is loaded lazily on first use.  There is no fallback: if the
shared library is missing or a tensor is not on a CUDA device, the call raises.
Every entry point is launched on the caller's current CUDA stream.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

import os

# GPA_LIB_PATH points the binding at another build of the same C ABI.
LIB_PATH = Path(os.environ.get("GPA_LIB_PATH") or Path(__file__).resolve().with_name("libgpa_b200.so"))

GPA_OK = 0
GPA_DTYPE_F32 = 0
GPA_DTYPE_BF16 = 1

_c_int = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_f32 = ctypes.c_float
_vp = ctypes.c_void_p

# name -> (restype, argtypes)
SIGNATURES = {
    "gpa_version": (_c_int, []),
    "gpa_last_error": (ctypes.c_char_p, []),
    "gpa_launch_count": (_c_i64, []),
    "gpa_wait_selftest": (_c_int, [ctypes.c_uint64, _vp, _vp]),
    "gpa_sim_argmax": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_i64, _c_i64,
                                _c_i64, _vp, _vp, _vp, _vp]),
    "gpa_merge_counts": (_c_int, [_c_int] * 7 + [ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "gpa_merge_roles": (_c_int, [_vp] + [_c_int] * 7 + [_vp, _vp, _vp, _vp]),
    "gpa_metric_split": (_c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _c_int, _vp, _c_int, _vp, _vp, _vp]),
    "gpa_proj_norm_split": (_c_int, [_vp, _c_i64, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gpa_merge_plan_workspace_bytes": (_c_i64, [_c_int, _c_int]),
    "gpa_merge_plan": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _c_i64, _vp]),
    "gpa_merge_plan_noalloc": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp]),
    "gpa_merge_kv_mean": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_i64, _vp, _vp, _vp,
                                   _c_int, _vp, _vp, _c_int, _c_int, _vp, _vp, _c_i64, _c_i64, _vp]),
    "gpa_ipc_export": (_c_int, [_vp, _vp, ctypes.POINTER(_c_i64)]),
    "gpa_ipc_open": (_c_int, [_vp, _c_i64, ctypes.POINTER(_vp)]),
    "gpa_ipc_close": (_c_int, [_vp, _c_i64]),
    "gpa_merge_exchange_p2p": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                        _c_int, _vp, _vp, _c_int, _c_int, _c_int, _vp, _vp]),
    "gpa_attention_keybias": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                       _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                       _c_i64, _c_i64, _c_i64, _c_f32, _vp, _c_i64, _c_i64, _c_i64,
                                       _vp, _c_i64, _c_i64, _vp, _vp]),
    "gpa_attention_keybias_combine": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                               _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                               _c_i64, _c_i64, _c_i64, _c_i64, _c_f32, _vp, _c_i64, _c_i64,
                                               _c_i64, _vp, _c_i64, _c_i64, _vp, _c_i64, _c_i64, _c_i64,
                                               _vp, _c_i64, _c_i64, _vp, _vp]),
    "gpa_layernorm_bf16": (_c_int, [_vp, _c_i64, _c_int, _c_int, _vp, _vp, _c_int, _c_f32, _vp, _c_i64, _vp]),
    "gpa_upsample_bilinear_bf16": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64, _c_i64,
                                            _c_i64, _vp, _c_i64, _c_i64, _c_int, _c_int, _c_int, _vp,
                                            _c_i64, _c_i64, _c_i64, _vp]),
    "gpa_gelu_bf16": (_c_int, [_vp, _c_i64, _vp, _vp]),
    "gpa_bias_act_bf16": (_c_int, [_vp, _vp, _vp, _c_i64, _c_int, _c_int, _vp, _vp]),
    "gpa_residual_scale_bf16": (_c_int, [_vp, _c_i64, _vp, _c_i64, _vp, _c_int, _c_int, _vp, _c_i64, _vp]),
    "gpa_qk_norm_rope": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                  _vp, _c_int, _c_f32, _vp, _vp, _vp, _c_int, _vp, _vp, _c_i64, _vp]),
    "gpa_frame_pool": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_i64,
                                _c_i64, _vp, _vp, _c_i64, _c_i64, _vp, _vp]),
    "gpa_lse_combine": (_c_int, [_c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


class GpaError(RuntimeError):
    """A C ABI call returned an error code."""


def load() -> ctypes.CDLL:
    """Load the shared library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m gpa_vggt_b200.build` "
                    "(there is no CPU or Triton fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != GPA_OK:
        msg = load().gpa_last_error().decode(errors="replace")
        raise GpaError(f"{what} failed (code {rc}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def ptr(t) -> _vp:
    if t is None:
        return _vp(0)
    return _vp(t.data_ptr())


def stream_of(t: torch.Tensor) -> _vp:
    return _vp(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors, what: str) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{what}: tensors must be on a CUDA device (no CPU fallback)")


def aligned(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def i64array(vals):
    arr = (_c_i64 * len(vals))(*[int(v) for v in vals])
    return arr


def launch_count() -> int:
    """Kernels launched by libgpa_b200 in this process so far."""
    return int(load().gpa_launch_count())
