"""Loading and registration of the XLA FFI targets (libalgx_jax.so), and the
host-only workspace queries of libalgx.so (no GPU needed for either)."""

from __future__ import annotations

import ctypes
import os
import threading

import jax

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIBDIR = os.path.join(os.path.dirname(_HERE), "algx")
TARGETS = {
    "algx_qknorm_fwd": "AlgxQkNormFwd",
    "algx_qknorm_bwd": "AlgxQkNormBwd",
    "algx_attn_fwd": "AlgxAttnFwd",
    "algx_attn_bwd": "AlgxAttnBwd",
    "algx_head_fwd": "AlgxHeadFwd",
    "algx_head_bwd": "AlgxHeadBwd",
}
_lock = threading.Lock()
_state = {}


def libs():
    """(libalgx, libalgx_jax), loaded once; the FFI targets are registered for CUDA."""
    with _lock:
        if not _state:
            core = ctypes.CDLL(os.path.join(_LIBDIR, "libalgx.so"))
            for name in ("algx_qknorm_bwd_workspace_size", "algx_attn_bwd_workspace_size",
                         "algx_head_bwd_workspace_size"):
                getattr(core, name).restype = ctypes.c_size_t
            core.algx_qknorm_bwd_workspace_size.argtypes = [ctypes.c_int64] * 2
            core.algx_attn_bwd_workspace_size.argtypes = [ctypes.c_int64] * 4
            core.algx_head_bwd_workspace_size.argtypes = [ctypes.c_int64] * 3 + [ctypes.c_int32]
            core.algx_head_fwd_splits.argtypes = [ctypes.c_int64] * 2
            core.algx_head_fwd_splits.restype = ctypes.c_int
            path = os.path.join(_LIBDIR, "libalgx_jax.so")
            if not os.path.exists(path):
                raise RuntimeError(f"{path} is missing: build it with jax_ffi/build.py (the algx kernels have no "
                                   "CPU fallback)")
            handlers = ctypes.CDLL(path)
            for target, symbol in TARGETS.items():
                jax.ffi.register_ffi_target(target, jax.ffi.pycapsule(getattr(handlers, symbol)), platform="CUDA")
            _state["libs"] = (core, handlers)
    return _state["libs"]


def core():
    return libs()[0]
