"""Element-type conversion without a GPU: the oracle against the reference's
known answer (test/ops_test.cpp:13-31) and against torch's CPU casts, and the
C ABI's argument checks (no kernel runs)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle.convert as oc
from llmx_b200 import _lib

TORCH = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def special_fp32():
    vals = [0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 65519.99, 70000.0, -1e30, 3.4e38, 6e-8, 5.96e-8, 2.98e-8,
            1e-40, -1e-45, 1.00390625, 1.0078125, 1.01171875, 0.1, 1 / 3, np.inf, -np.inf]
    g = np.random.default_rng(0)
    scaled = (g.standard_normal(20000) * 10.0 ** g.integers(-8, 8, 20000)).astype(np.float32)
    patterns = g.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([np.array(vals, dtype=np.float32), scaled, patterns])
    return x


def as_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.numpy().copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(b: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "fp32":
        return torch.from_numpy(np.asarray(b, np.float32).copy())
    return torch.from_numpy(np.asarray(b, np.uint16).view(np.int16).copy()).view(TORCH[dtype])


def test_reference_known_answer_fp16_to_fp32():
    # ops_test.cpp: fp16 [1, 2, 3, 4] -> to_fp32 -> [1, 2, 3, 4]
    src = np.array([1, 2, 3, 4], dtype=np.float16).view(np.uint16)
    out = oc.convert(src, "fp16", "fp32")
    assert out.dtype == np.float32 and out.tolist() == [1.0, 2.0, 3.0, 4.0]


@pytest.mark.parametrize("src", oc.DTYPES)
@pytest.mark.parametrize("dst", oc.DTYPES)
def test_oracle_matches_torch_cpu_casts(src, dst):
    x = torch.from_numpy(special_fp32())
    xs = x.to(TORCH[src])  # inputs of the source type (torch rounds fp32 -> src once)
    want = xs.to(TORCH[dst])
    got = from_bits(oc.convert(as_bits(xs), src, dst), dst)
    nan = torch.isnan(want.float())
    assert torch.equal(torch.isnan(got.float()), nan)
    keep = ~nan.numpy()
    assert np.array_equal(as_bits(got)[keep].view(np.uint32 if dst == "fp32" else np.uint16),
                          as_bits(want)[keep].view(np.uint32 if dst == "fp32" else np.uint16))


def test_bf16_ties_round_to_even():
    # 1 + 2^-8 is halfway between bf16 1.0 and 1.0078125: rounds to the even 1.0;
    # 1 + 3 * 2^-8 is halfway between 1.0078125 and 1.015625: rounds up.
    b = oc.from_float32(np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8], np.float32), "bf16")
    assert oc.to_float32(b, "bf16").tolist() == [1.0, 1.015625]


def test_abi_argument_checks_need_no_gpu():
    lib = _lib.load()
    buf = (ctypes.c_char * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.llmx_convert(p, 7, p, 0, 4, None) == 1
    assert lib.llmx_convert(p, 0, p, -1, 4, None) == 1
    assert lib.llmx_convert(None, 0, p, 1, 4, None) == 1
    assert lib.llmx_convert(None, 0, None, 1, 0, None) == 0  # nothing to do
    # A pageable host buffer is refused (or, without a device, the device query fails).
    assert lib.llmx_convert(p, 0, p, 1, 4, None) != 0
