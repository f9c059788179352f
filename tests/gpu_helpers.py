"""Shared helpers for the GPU parity tests: tolerances and oracle calls.

Tolerances (stated once, used by every GPU test):
  * fp32 outputs: max-abs error <= 1e-4 against the fp32 oracle;
  * fp16 / bf16 outputs: max-abs error <= 2e-2 and mean-relative error
    (mean |out - ref| / mean |ref|) <= 1e-2 against the fp32 oracle.
"""
import numpy as np
import pytest
import torch

import oracle

FP32_MAX_ABS = 1e-4
HALF_MAX_ABS = 2e-2
HALF_MEAN_REL = 1e-2

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def assert_close(out: torch.Tensor, ref: torch.Tensor, dtype, what: str = "") -> dict:
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert o.shape == r.shape, (o.shape, r.shape)
    assert torch.isfinite(o).all(), f"{what}: non-finite output"
    err = (o - r).abs()
    max_abs = float(err.max()) if err.numel() else 0.0
    mean_rel = float(err.mean() / r.abs().mean().clamp_min(1e-12)) if err.numel() else 0.0
    if dtype == torch.float32:
        assert max_abs <= FP32_MAX_ABS, f"{what}: max-abs {max_abs:.3e} > {FP32_MAX_ABS}"
    else:
        assert max_abs <= HALF_MAX_ABS, f"{what}: max-abs {max_abs:.3e} > {HALF_MAX_ABS}"
        assert mean_rel <= HALF_MEAN_REL, f"{what}: mean-rel {mean_rel:.3e} > {HALF_MEAN_REL}"
    return {"max_abs": max_abs, "mean_rel": mean_rel}


def assert_close_np(got: np.ndarray, ref: np.ndarray, dtype, what: str = "") -> None:
    assert_close(torch.from_numpy(got), torch.from_numpy(ref), dtype, what)


def oracle_fp32(q, k, v, **kw):
    """Oracle output kept in fp32 (no final cast) for single sequences."""
    return oracle.attention_ref(q.float().cpu(), k.float().cpu(), v.float().cpu(), **kw)


def oracle_padded_fp32(q, k, v, **kw):
    return oracle.attention_ref_padded(q.float().cpu(), k.float().cpu(), v.float().cpu(), **kw)
