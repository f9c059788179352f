"""llmx_b200: B200-native (sm_100a) fused attention forward for llmx.

The compute lives in libllmx_attn.so (CUDA, C ABI in include/llmx_attn.h);
this package is the torch-facing host side.  The library is loaded on first
use and every op raises if it has not been built -- there is no fallback
path.  Build it with `python -m llmx_b200.build`.
"""
from ._lib import LlmxError, load  # noqa: F401
from .ops import attention, convert, device_status, selected_algo, single_mha_attention_half  # noqa: F401
from .streaming import HostAttention, attention_from_host  # noqa: F401

__all__ = ["single_mha_attention_half", "attention", "convert", "selected_algo", "device_status", "LlmxError",
           "load", "HostAttention", "attention_from_host"]
