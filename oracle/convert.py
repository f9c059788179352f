"""CPU oracle for llmx's element-type conversion (to_fp32 / to_fp16 / to_bf16).

TEST INFRASTRUCTURE ONLY, like the rest of this package: only ``tests/`` may
import it, as the checker.  The product path (``llmx_b200.convert`` and the
library's ``llmx_convert``) never calls it.

Restates the reference's scalar conversion (src/scalar.cu:6-46, reached via
llmx_copy, src/tensor.cpp:108-118, from the operators in
include/llmx/ops.h:25-74):

* fp32 -> fp16 / bf16: round to nearest, ties to even (``__float2half`` /
  ``__float2bfloat16``, scalar.cu:8-15); overflow goes to +-inf, fp16
  subnormals are kept.
* fp16 / bf16 -> fp32: exact widening (scalar.cu:17-24).
* fp16 <-> bf16: through fp32 (scalar.cu:26-31), so one rounding.
* same type: the reference's converter is a no-op (include/llmx/scalar.h:13-15);
  the library copies, so the oracle returns the input bits.

Values travel as raw bit patterns (uint16 for the 16-bit types, float32
otherwise).  fp16 rounding is numpy's IEEE conversion; bf16 rounding is the
usual integer form of round-to-nearest-even on the upper 16 bits of the
fp32 pattern (add 0x7FFF plus the lowest kept bit, truncate), with NaNs
mapped to a quiet NaN of the same sign.

Pinned by the reference's own known answer (test/ops_test.cpp:13-31: fp16
[1, 2, 3, 4] -> fp32 [1, 2, 3, 4]) and by the CPU casts of torch in
tests/test_convert.py.
"""

from __future__ import annotations

import numpy as np

DTYPES = ("fp32", "fp16", "bf16")


def to_float32(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Exact fp32 values of raw `dtype` bit patterns."""
    if dtype == "fp32":
        return np.asarray(bits, dtype=np.float32)
    b = np.asarray(bits, dtype=np.uint16)
    if dtype == "fp16":
        return b.view(np.float16).astype(np.float32)
    if dtype == "bf16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    raise ValueError(dtype)


def from_float32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Raw `dtype` bit patterns of fp32 values, round to nearest even."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x.copy()
    if dtype == "fp16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        nan = np.isnan(x)
        quiet = ((u >> 16) | 0x0040).astype(np.uint16)
        return np.where(nan, quiet, rounded).astype(np.uint16)
    raise ValueError(dtype)


def convert(bits: np.ndarray, src: str, dst: str) -> np.ndarray:
    """`bits` of type `src` converted to `dst` (raw patterns in and out)."""
    if src == dst:
        return np.array(bits, copy=True)
    return from_float32(to_float32(bits, src), dst)
