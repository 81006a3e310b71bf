"""ctypes binding of libalgx.so (the C ABI declared in include/algx.h).

The library is built in-tree next to this file. Loading fails loudly when it
is missing; there is no CPU fallback anywhere in the package.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libalgx.so")

ALGX_OK, ALGX_ERR_INVALID, ALGX_ERR_UNSUPPORTED, ALGX_ERR_CUDA = 0, 1, 2, 3
ALGX_F32, ALGX_BF16 = 0, 1
ALGX_ATTN_ASINH, ALGX_ATTN_SOFTMAX = 0, 1
ALGX_MODE_CLIPPED, ALGX_MODE_SHIFTED, ALGX_MODE_GUARDED = 0, 1, 2
ALGX_HEAD_CE, ALGX_HEAD_ALG_CE = 0, 1


class AlgxError(RuntimeError):
    """A libalgx call returned a non-zero status."""


class AttnConfig(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("fast_rho", ctypes.c_int32),
        ("inv_stat", ctypes.c_int32),
        ("has_sink", ctypes.c_int32),
        ("clamp", ctypes.c_float),
        ("scale", ctypes.c_float),
        ("guard_qk", ctypes.c_float),
        ("guard_sink", ctypes.c_float),
        ("guard_v", ctypes.c_float),
    ]


class HeadConfig(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("inv_c", ctypes.c_float),
        ("clamp", ctypes.c_float),
        ("has_ignore", ctypes.c_int32),
        ("ignore_index", ctypes.c_int32),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_SZ = ctypes.c_size_t

SIGNATURES = {
    "algx_last_error": ([], ctypes.c_char_p),
    "algx_version": ([], ctypes.c_int),
    "algx_launch_count": ([], ctypes.c_uint64),
    "algx_device_error": ([ctypes.POINTER(_I32)], ctypes.c_int),
    "algx_qknorm_fwd": ([_P, _P, _P, _I64, _I64, _I32, _F, _P], ctypes.c_int),
    "algx_qknorm_bwd_workspace_size": ([_I64, _I64], _SZ),
    "algx_qknorm_bwd": ([_P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _P, _SZ, _P], ctypes.c_int),
    "algx_qknorm_bwd_noalloc": ([_P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _P], ctypes.c_int),
    "algx_attn_prepare": ([ctypes.POINTER(AttnConfig), _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
                          ctypes.c_int),
    "algx_qknorm_attn_prepare": ([ctypes.POINTER(AttnConfig)] + [_P] * 7 + [_I64] + [_P] * 4 +
                                 [_I64, _I64, _I64, _I64, _I32, _F, _P], ctypes.c_int),
    "algx_attn_fwd": ([ctypes.POINTER(AttnConfig), _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _P],
                      ctypes.c_int),
    "algx_attn_bwd_workspace_size": ([_I64, _I64, _I64, _I64], _SZ),
    "algx_attn_bwd": ([ctypes.POINTER(AttnConfig), _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                       _I64, _I64, _I64, _I64, _I32, _P, _SZ, _P], ctypes.c_int),
    "algx_qknorm_attn_bwd_workspace_size": ([_I64, _I64, _I64, _I64], _SZ),
    "algx_qknorm_attn_bwd": ([ctypes.POINTER(AttnConfig)] + [_P] * 6 + [_I64] + [_P] * 15 +
                             [_I64, _I64, _I64, _I64, _I32, _F, _P, _SZ, _P], ctypes.c_int),
    "algx_head_fwd_splits": ([_I64, _I64], ctypes.c_int),
    "algx_head_fwd": ([ctypes.POINTER(HeadConfig), _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _P],
                      ctypes.c_int),
    "algx_head_reduce": ([ctypes.POINTER(HeadConfig), _P, _P, _P, _I32, _I64, _P, _P, _P, _P], ctypes.c_int),
    "algx_head_finalize": ([ctypes.POINTER(HeadConfig), _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _P],
                           ctypes.c_int),
    "algx_head_bwd_workspace_size": ([_I64, _I64, _I64, _I32], ctypes.c_size_t),
    "algx_head_bwd": ([ctypes.POINTER(HeadConfig), _P, _P, _P, _P, _P, _P, _I32, _P, _I64, _I64, _I64, _I64, _I32,
                       _P, ctypes.c_size_t, _P], ctypes.c_int),
    "algx_qknorm_attn_prepare_packed": ([ctypes.POINTER(AttnConfig)] + [_P] * 5 + [_I64] + [_P] * 5 +
                                        [_I64, _I64, _I64, _I64, _I32, _F, _P], ctypes.c_int),
    "algx_qknorm_attn_bwd_packed_workspace_size": ([_I64, _I64, _I64, _I64, _I32], _SZ),
    "algx_qknorm_attn_bwd_packed": ([ctypes.POINTER(AttnConfig)] + [_P] * 5 + [_I64] + [_P] * 13 +
                                    [_I64, _I64, _I64, _I64, _I32, _F, _P, _SZ, _P], ctypes.c_int),
    "algx_heads_to_tokens": ([_P, _P, _I64, _I64, _I64, _I64, _I32, _P], ctypes.c_int),
    "algx_tokens_to_heads": ([_P, _P, _I64, _I64, _I64, _I64, _I32, _P], ctypes.c_int),
    "algx_rmsnorm_fwd": ([_P, _P, _P, _I64, _I64, _I32, _F, _P], ctypes.c_int),
    "algx_rmsnorm_bwd_workspace_size": ([_I64, _I64], _SZ),
    "algx_rmsnorm_bwd": ([_P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _P, _SZ, _P], ctypes.c_int),
    "algx_add_rmsnorm_fwd": ([_P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _P], ctypes.c_int),
    "algx_add_rmsnorm_bwd": ([_P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _F, _P, _SZ, _P], ctypes.c_int),
    "algx_swiglu_fwd": ([_P, _P, _I64, _I64, _P], ctypes.c_int),
    "algx_swiglu_bwd": ([_P, _P, _P, _I64, _I64, _P], ctypes.c_int),
    "algx_aluglu_fwd": ([_P, _P, _I64, _I64, _F, _P], ctypes.c_int),
    "algx_aluglu_bwd": ([_P, _P, _P, _I64, _I64, _F, _P], ctypes.c_int),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load libalgx.so once; raise if it is missing (no fallback exists)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise AlgxError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                                    "(the algx kernels have no CPU fallback)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (args, res) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != ALGX_OK:
        msg = lib().algx_last_error().decode(errors="replace")
        kind = {ALGX_ERR_INVALID: "invalid argument", ALGX_ERR_UNSUPPORTED: "unsupported",
                ALGX_ERR_CUDA: "CUDA error"}.get(status, f"status {status}")
        raise AlgxError(f"{what}: {kind}: {msg}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise AlgxError("algx kernels run on CUDA tensors only (no CPU fallback); got a tensor on "
                            f"{t.device}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return ALGX_BF16
    if dt == torch.float32:
        return ALGX_F32
    raise ValueError(f"unsupported dtype {dt}")


def device_error() -> int:
    """Read and clear the device error word (synchronizes)."""
    code = _I32(0)
    check(lib().algx_device_error(ctypes.byref(code)), "algx_device_error")
    return int(code.value)
