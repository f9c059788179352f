"""ctypes view of the C ABI in include/llmx_attn.h (libllmx_attn.so).

The library is built in-tree (``python -m llmx_b200.build``).  Loading fails
loudly when it is missing: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libllmx_attn.so")

LLMX_OK = 0
STATUS_NAMES = {
    0: "LLMX_OK",
    1: "LLMX_ERR_INVALID_ARGUMENT",
    2: "LLMX_ERR_UNSUPPORTED",
    3: "LLMX_ERR_WORKSPACE_TOO_SMALL",
    4: "LLMX_ERR_CUDA",
    5: "LLMX_ERR_TIMEOUT",
    6: "LLMX_ERR_NO_DEVICE",
}
DTYPE = {"fp32": 0, "fp16": 1, "bf16": 2}
ALGO = {"auto": 0, "simt": 1, "decode": 2, "tcgen05": 3}
ALGO_NAMES = {v: k for k, v in ALGO.items()}

_i32 = ctypes.c_int32
_i64x3 = ctypes.c_int64 * 3
_vp = ctypes.c_void_p


class AttnParams(ctypes.Structure):
    """Mirror of ``llmx_attn_params``."""

    _fields_ = [
        ("dtype", _i32),
        ("batch", _i32),
        ("n_heads", _i32),
        ("n_kv_heads", _i32),
        ("head_dim", _i32),
        ("max_q_len", _i32),
        ("max_kv_len", _i32),
        ("algo", _i32),
        ("q", _vp),
        ("k", _vp),
        ("v", _vp),
        ("o", _vp),
        ("q_stride", _i64x3),
        ("k_stride", _i64x3),
        ("v_stride", _i64x3),
        ("o_stride", _i64x3),
        ("q_lens", _vp),
        ("kv_lens", _vp),
        ("alibi_slopes", _vp),
        ("sm_scale", ctypes.c_float),
        ("causal", _i32),
        ("sliding_window", _i32),
        ("logits_soft_cap", ctypes.c_float),
        ("lse", _vp),
        ("workspace", _vp),
        ("workspace_bytes", ctypes.c_size_t),
        ("kv_offset", _i32),
        ("kv_total", _i32),
    ]


class MergePart(ctypes.Structure):
    """Mirror of ``llmx_merge_part``."""

    _fields_ = [
        ("o", _vp),
        ("lse", _vp),
        ("o_stride", _i64x3),
        ("lse_stride", ctypes.c_int64 * 2),
        ("row_lo", _i32),
        ("row_hi", _i32),
    ]


class RowScatter(ctypes.Structure):
    """Mirror of ``llmx_row_scatter``."""

    _fields_ = [
        ("n_dst", _i32),
        ("slice_rows", _i32),
        ("row_base", _i32),
        ("reserved", _i32),
        ("o", _vp * 8),
        ("lse", _vp * 8),
    ]


IPC_HANDLE_BYTES = 64

# Every function include/llmx_attn.h declares: name -> (restype, argtypes).
SIGNATURES = {
    "llmx_attn_params_init": (_i32, [ctypes.POINTER(AttnParams)]),
    "llmx_attn_set_contiguous_strides": (_i32, [ctypes.POINTER(AttnParams)]),
    "llmx_attn_workspace_size": (_i32, [ctypes.POINTER(AttnParams), ctypes.POINTER(ctypes.c_size_t)]),
    "llmx_attn_fwd": (_i32, [ctypes.POINTER(AttnParams), _vp]),
    "llmx_single_mha_attention_c": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.c_float, _i32, ctypes.c_float, _vp],
    ),
    "llmx_attn_select_algo": (_i32, [ctypes.POINTER(AttnParams), ctypes.POINTER(_i32)]),
    "llmx_attn_decode_noalloc": (_i32, [ctypes.POINTER(AttnParams), _vp]),
    "llmx_attn_lse_merge": (
        _i32,
        [_i32, ctypes.POINTER(MergePart), _i32, _i32, _i32, _i32, _i32, _vp, ctypes.POINTER(ctypes.c_int64), _vp,
         _vp],
    ),
    "llmx_attn_fwd_scatter": (_i32, [ctypes.POINTER(AttnParams), ctypes.POINTER(RowScatter), _vp]),
    "llmx_ipc_alloc": (_i32, [ctypes.c_size_t, ctypes.POINTER(_vp), _vp]),
    "llmx_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "llmx_ipc_close": (_i32, [_vp]),
    "llmx_ipc_free": (_i32, [_vp]),
    "llmx_convert": (_i32, [_vp, _i32, _vp, _i32, ctypes.c_size_t, _vp]),
    "llmx_attn_device_status": (_i32, [_i32, _i32]),
    "llmx_status_string": (ctypes.c_char_p, [_i32]),
    "llmx_attn_last_error": (ctypes.c_char_p, []),
    "llmx_attn_abi_version": (_i32, []),
}

_LIB = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads (once) and types the library; raises if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise ImportError(
            f"llmx_b200: {path} is missing; build it with `python -m llmx_b200.build` "
            "(there is no fallback implementation)"
        )
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class LlmxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def check(status: int) -> None:
    if status != LLMX_OK:
        msg = load().llmx_attn_last_error()
        raise LlmxError(status, msg.decode() if msg else "")
