"""Element-type conversion on the GPU through the C ABI (llmx_convert, via
llmx_b200.convert): bit-exact against the oracle (NaN positions compared as
NaN), on aligned and unaligned buffers, ragged sizes and a size-independent
round-trip property at 256 Mi elements."""
import numpy as np
import pytest
import torch

import llmx_b200
import oracle.convert as oc
from gpu_helpers import needs_cuda

pytestmark = [pytest.mark.gpu, needs_cuda]

TORCH = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.cpu()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy().view(np.uint32).copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()


def inputs(n: int, dtype: str, seed: int) -> torch.Tensor:
    g = np.random.default_rng(seed)
    specials = np.array([0.0, -0.0, 1.0, 65504.0, 65520.0, 70000.0, 3.4e38, 6e-8, 2.98e-8, 1e-40, np.inf,
                         -np.inf, np.nan, 1.00390625, 1.01171875], np.float32)
    mixed = np.concatenate([
        (g.standard_normal(n) * 10.0 ** g.integers(-8, 8, n)).astype(np.float32),
        g.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32).view(np.float32),
    ])
    x = np.resize(np.concatenate([specials, mixed[: 2 * n]]), n)
    return torch.from_numpy(x).to(TORCH[dtype])


def check(src: torch.Tensor, out: torch.Tensor, s: str, d: str):
    want = oc.convert(bits(src).view(np.float32) if s == "fp32" else bits(src), s, d)
    want = want.view(np.uint32) if d == "fp32" else want
    got = bits(out)
    wf = oc.to_float32(want.view(np.float32) if d == "fp32" else want, d)
    nan = np.isnan(wf)
    assert np.array_equal(np.isnan(oc.to_float32(got.view(np.float32) if d == "fp32" else got, d)), nan)
    assert np.array_equal(got[~nan], want[~nan]), f"{s}->{d}: {(got[~nan] != want[~nan]).sum()} mismatches"


@pytest.mark.parametrize("s", oc.DTYPES)
@pytest.mark.parametrize("d", oc.DTYPES)
@pytest.mark.parametrize("n", [1, 7, 8, 1003, 65536 * 3 + 5])
def test_convert_matches_oracle(s, d, n):
    src = inputs(n, s, seed=n).cuda()
    out = llmx_b200.convert(src, TORCH[d])
    torch.cuda.synchronize()
    check(src, out, s, d)


@pytest.mark.parametrize("s,d", [("fp32", "bf16"), ("fp16", "fp32"), ("bf16", "fp16")])
def test_unaligned_views_take_the_scalar_path(s, d):
    base = inputs(4099, s, seed=3).cuda()
    src = base[1:]  # 2- or 4-byte offset: not 16-byte aligned
    out_base = torch.empty(4099, dtype=TORCH[d], device="cuda")
    out = out_base[3:]
    llmx_b200.convert(src[:4096], TORCH[d], out=out[:4096])
    torch.cuda.synchronize()
    check(src[:4096], out[:4096], s, d)


def test_reference_known_answer():
    # test/ops_test.cpp: fp16 [1, 2, 3, 4] -> fp32 [1, 2, 3, 4]
    out = llmx_b200.convert(torch.tensor([1, 2, 3, 4], dtype=torch.float16, device="cuda"), torch.float32)
    assert out.cpu().tolist() == [1.0, 2.0, 3.0, 4.0]


def test_large_round_trip_is_exact():
    # bf16 -> fp32 -> bf16 and fp16 -> fp32 -> fp16 are identities (widening is
    # exact); fp32 -> bf16 -> fp32 -> bf16 is idempotent.  256 Mi elements.
    n = 256 << 20
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(n, generator=g, device="cuda")
    b = llmx_b200.convert(x, torch.bfloat16)
    w = llmx_b200.convert(b, torch.float32)
    b2 = llmx_b200.convert(w, torch.bfloat16)
    assert torch.equal(b.view(torch.int16), b2.view(torch.int16))
    assert torch.equal(b.view(torch.int16), x.to(torch.bfloat16).view(torch.int16))
    h = llmx_b200.convert(b, torch.float16)
    assert torch.equal(h.view(torch.int16), b.to(torch.float16).view(torch.int16))
    del x, w, b2
    hw = llmx_b200.convert(h, torch.float32)
    assert torch.equal(llmx_b200.convert(hw, torch.float16).view(torch.int16), h.view(torch.int16))


def test_host_buffers_are_refused():
    host = torch.ones(64)
    with pytest.raises(llmx_b200.LlmxError):
        from llmx_b200 import _lib
        import ctypes
        _lib.check(_lib.load().llmx_convert(ctypes.c_void_p(host.data_ptr()), 0, ctypes.c_void_p(host.data_ptr()),
                                            1, 64, None))
