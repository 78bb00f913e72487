"""ctypes binding of the in-tree C-ABI library ``libogx.so`` (declared in include/ogx.h).

The library is the only compute path: when it is missing or fails to load, every
op raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_uint, c_void_p

LIB_NAME = "libogx.so"
# OPENGENIE_B200_LIB selects another build of the same library (e.g. a tuning variant).
LIB_PATH = os.environ.get("OPENGENIE_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

OGX_OK = 0
DTYPE_BF16 = 0
DTYPE_F32 = 1
DTYPE_F16 = 2
QUANT_TORCH = 0
QUANT_SINGLE = 1

# name -> argument types (restype is c_int for all entry points but ogx_last_error)
_SIGNATURES: dict[str, list] = {
    "ogx_version": [],
    "ogx_device_status": [ctypes.POINTER(c_uint), c_int],
    "ogx_adazero_from_ada": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int,
        c_int64, c_int64, c_int64, c_int, c_int, c_float, c_void_p, c_void_p,
    ],
    "ogx_head_gate_mul_bf16": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p],
    "ogx_mul_from_ada": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int,
        c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p,
    ],
    "ogx_adaln_affine_from_ada": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int,
        c_int64, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p,
    ],
    "ogx_adazero_from_ada_e4m3": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int,
        c_int64, c_int64, c_int64, c_int, c_int, c_float, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
    ],
    "ogx_adazero_from_ada_e4m3_planes": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int,
        c_int64, c_int64, c_int64, c_int, c_int, c_float, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int64, c_void_p,
    ],
    "ogx_fp8_quantize_e4m3": [c_void_p, c_int, c_int64, c_void_p, c_int, c_void_p, c_void_p],
    "ogx_bias_add_bf16": [c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p, c_void_p],
    "ogx_residual_gate_bias_from_ada": [
        c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_int, c_int64,
        c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p,
    ],
    "ogx_video_qk_rmsnorm_rope": [
        c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p, c_void_p,
        c_int, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
    ],
    "ogx_video_qk_rmsnorm_rope_positions": [
        c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p, c_void_p,
        c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
    ],
    "ogx_video_qkv_rmsnorm_rope_positions_scatter": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p,
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p,
    ],
    "ogx_rope_tables_from_positions": [
        c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p, c_void_p,
    ],
    "ogx_video_qkv_rmsnorm_rope_scatter": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p,
        c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p,
    ],
    "ogx_fp8_scaled_mm": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
        c_void_p, c_int, c_void_p, c_int64, c_void_p,
    ],
    "ogx_fp8_scaled_mm_planes": [
        c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
        c_void_p, c_int, c_void_p, c_int64, c_void_p,
    ],
    "ogx_fp8_scaled_mm_residual_gate": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int, c_int64, c_int64,
        c_int, c_void_p, c_int64, c_void_p,
    ],
    "ogx_fp8_scaled_mm_residual_gate_kblocked": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int, c_int64, c_int64,
        c_int, c_void_p, c_int64, c_void_p,
    ],
    "ogx_attention_fwd": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_float,
        c_void_p, c_int64, c_int64, c_void_p,
    ],
    "ogx_attention_fwd_e4m3": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_float,
        c_void_p, c_void_p, c_int64, c_int64, c_void_p,
    ],
    "ogx_attention_fwd_kv": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
        c_int64, c_int64, c_float, c_void_p, c_int64, c_int64, c_void_p,
    ],
    "ogx_attention_fwd_kv_e4m3": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
        c_int64, c_int64, c_float, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
    ],
    "ogx_qk_rmsnorm": [
        c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float,
        c_void_p, c_int64, c_void_p, c_int64, c_void_p,
    ],
    "ogx_ipc_get_handle": [c_void_p, c_void_p, ctypes.POINTER(c_int64)],
    "ogx_ipc_open_handle": [c_void_p, ctypes.POINTER(c_void_p)],
    "ogx_ipc_close_handle": [c_void_p],
    "ogx_peer_barrier": [c_void_p, c_void_p, c_int, c_int, c_void_p],
    "ogx_gelu_tanh_fp8_quantize_e4m3": [c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "ogx_fp8_scaled_mm_gelu_e4m3": [
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
        c_void_p, c_int, c_void_p, c_void_p, c_int64, c_void_p,
    ],
    "ogx_peer_barrier_static": [c_int, c_int, c_void_p, c_void_p, c_void_p],
    "ogx_video_qkv_rmsnorm_rope_to_peers": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p,
        c_void_p, c_int, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p,
    ],
    "ogx_video_qkv_rmsnorm_rope_positions_to_peers": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int, c_float, c_void_p,
        c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int64, c_void_p,
    ],
    "ogx_attention_fwd_e4m3_to_peers": [
        c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_float, c_void_p, c_void_p, c_int, c_int64,
        c_int64, c_void_p,
    ],
}

EXPORTED = tuple(sorted(list(_SIGNATURES) + ["ogx_last_error"]))

_LIB: ctypes.CDLL | None = None


class OgxError(RuntimeError):
    """A C-ABI call returned an error; the message is ogx_last_error()."""


def load() -> ctypes.CDLL:
    """Loads libogx.so from the package directory (built by ``opengenie_b200.build``)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import opengenie_b200.build as b; b.build()'` "
            "(there is no fallback compute path)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = c_int
    lib.ogx_last_error.argtypes = []
    lib.ogx_last_error.restype = ctypes.c_char_p
    _LIB = lib
    return lib


def call(name: str, *args) -> None:
    """Calls an entry point and raises OgxError (reason string from the library) on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OGX_OK:
        msg = lib.ogx_last_error().decode(errors="replace")
        raise OgxError(f"{name}: {msg}" if msg else f"{name}: error {rc}")


OGX_ERR_TIMEOUT = 1  # device status bit: a bounded device-side wait gave up


def device_status(clear: bool = True) -> int:
    """Device status word (bit OGX_ERR_TIMEOUT: a bounded device-side wait timed out)."""
    lib = load()
    v = c_uint(0)
    rc = lib.ogx_device_status(ctypes.byref(v), 1 if clear else 0)
    if rc != OGX_OK:
        raise OgxError(lib.ogx_last_error().decode(errors="replace"))
    return int(v.value)
