"""llmx_b200: B200-native (sm_100a) fused attention forward for llmx.

The compute lives in libllmx_attn.so (CUDA, C ABI in include/llmx_attn.h);
this package is the torch-facing host side.  Importing it loads the library
and fails if it has not been built -- there is no fallback path.
"""
from . import _lib

_lib.load()

from .ops import attention, device_status, selected_algo, single_mha_attention_half  # noqa: E402,F401
from ._lib import LlmxError  # noqa: E402,F401

__all__ = ["single_mha_attention_half", "attention", "selected_algo", "device_status", "LlmxError"]
