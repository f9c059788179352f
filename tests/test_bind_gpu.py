"""The torch bindings on the GPU against the golden fixtures.

* llmx_b200.llmx_bind (this repository's C++ torch binding,
  llmx_b200/csrc/llmx_bind.cpp): every golden case, on torch's current
  stream, against the stored ref_attention outputs and the fp32 oracle;
* the reference's own binding source (csrc/llmx_bind.cpp) and C++ smoke
  test (test/cuda/mha_attention_test.cpp), compiled unchanged against
  include/ + libllmx_attn.so by oracle/build_ref_boundary.py: the smoke test
  runs to "done", and the binding runs the reference's 16-case parity suite
  (csrc/test_attention.py:143-201; one causal sequence, fp16/bf16, no ALiBi:
  what its signature takes).  Skipped when those files were not built.
Tolerances: see gpu_helpers.
"""
import importlib.util
import os
import subprocess

import pytest
import torch

from cases import make_inputs
from golden_io import load_golden
from gpu_helpers import assert_close, assert_close_np, needs_cuda, oracle_fp32, oracle_padded_fp32

pytestmark = [pytest.mark.gpu, needs_cuda]

CASES = load_golden()


def _bind():
    from llmx_b200 import build as b

    b.build_binding()
    import llmx_b200.llmx_bind as m

    return m


@pytest.mark.parametrize("case", CASES, ids=[c[0].name for c in CASES])
def test_cpp_binding_golden(case):
    m = _bind()
    c, entry, idx, val = case
    q, k, v, slopes = make_inputs(c)
    dev = torch.device("cuda", 0)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out = torch.full_like(qd, float("nan"))
    kw = dict(alibi_slopes=None if slopes is None else slopes.to(dev), causal=c.causal)
    if c.kind == "padded":
        if c.q_lens:
            kw["q_lens"] = torch.tensor(c.q_lens, dtype=torch.int32, device=dev)
        if c.kv_lens:
            kw["kv_lens"] = torch.tensor(c.kv_lens, dtype=torch.int32, device=dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):  # the binding runs on torch's current stream
        m.single_mha_attention_half(out, qd, kd, vd, c.sm_scale, c.sliding_window, c.logits_soft_cap, **kw)
    s.synchronize()
    got = out.float().cpu().reshape(-1).numpy()
    assert_close_np(got[idx], val, q.dtype, f"{c.name} via llmx_bind vs golden")
    okw = dict(sm_scale=c.sm_scale, logits_soft_cap=c.logits_soft_cap, sliding_window=c.sliding_window,
               alibi=slopes, causal=c.causal)
    ref = (oracle_fp32(q, k, v, **okw) if c.kind == "single"
           else oracle_padded_fp32(q, k, v, q_lens=c.q_lens, kv_lens=c.kv_lens, **okw))
    assert_close(out, ref, q.dtype, f"{c.name} via llmx_bind vs oracle")


def _ref_artifacts():
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("build_ref_boundary",
                                                  os.path.join(here, "..", "oracle", "build_ref_boundary.py"))
    rb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rb)
    return rb.ref_binding_path(), rb.ref_test_path()


def test_reference_cpp_smoke_test_runs_against_this_library():
    _, exe = _ref_artifacts()
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/mha_attention_test not built (needs the reference source)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "done" in r.stdout


REF_SUITE = [c for c in CASES if c[0].kind == "single" and c[0].dtype in ("fp16", "bf16") and not c[0].alibi
             and c[0].causal and c[0].q_len <= c[0].kv_len]


@pytest.mark.parametrize("case", REF_SUITE, ids=[c[0].name for c in REF_SUITE])
def test_reference_binding_source_golden(case):
    so, _ = _ref_artifacts()
    if not os.path.exists(so):
        pytest.skip("oracle/_ref/llmx_ref_bind not built (needs the reference source)")
    spec = importlib.util.spec_from_file_location("llmx_ref_bind", so)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    c, entry, idx, val = case
    q, k, v, _ = make_inputs(c)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    out = torch.full_like(qd, float("nan"))
    m.single_mha_attention_half(out, qd, kd, vd, c.sm_scale, c.sliding_window, c.logits_soft_cap)
    torch.cuda.synchronize()
    got = out.float().cpu().reshape(-1).numpy()
    assert_close_np(got[idx], val, q.dtype, f"{c.name} via the reference's binding vs golden")


@pytest.mark.parametrize("shape,dtype,kw", [
    ((2, 300, 8, 128), torch.bfloat16, dict(causal=True)),
    ((3, 1, 8, 128), torch.float16, dict(kv_len=700)),
    ((1, 128, 8, 64), torch.float32, dict(causal=True)),
])
def test_binding_and_ctypes_routes_agree_bitwise(shape, dtype, kw):
    import llmx_b200
    from llmx_b200 import ops

    _bind()
    B, S, H, D = shape
    g = torch.Generator().manual_seed(5)
    Skv = kw.get("kv_len", S)
    q = torch.randn(B, S, H, D, generator=g).to(dtype).cuda()
    k = torch.randn(B, Skv, H // 2, D, generator=g).to(dtype).cuda()
    v = torch.randn(B, Skv, H // 2, D, generator=g).to(dtype).cuda()
    slopes = torch.pow(2.0, -8.0 * torch.arange(1, H + 1) / H).float().cuda()
    lens = torch.tensor([Skv - 37 * b for b in range(B)], dtype=torch.int32).cuda()
    a, b_ = torch.empty_like(q), torch.empty_like(q)
    la, lb = torch.empty(B, H, S).cuda(), torch.empty(B, H, S).cuda()
    args = dict(alibi_slopes=slopes, causal=kw.get("causal", True), kv_lens=lens)
    llmx_b200.single_mha_attention_half(a, q, k, v, D ** -0.5, lse=la, **args)
    ops.single_mha_attention_half_ctypes(b_, q, k, v, D ** -0.5, lse=lb, **args)
    torch.cuda.synchronize()
    assert torch.equal(a, b_) and torch.equal(la, lb)
    # library failures come back as LlmxError(status) on both routes
    # (forcing a kernel family that cannot run the request: decode for a prefill, tcgen05 for fp32)
    bad = "tcgen05" if dtype == torch.float32 else ("decode" if S > 1 else None)
    for fn in (llmx_b200.single_mha_attention_half, ops.single_mha_attention_half_ctypes):
        if bad is None:
            continue
        with pytest.raises(llmx_b200.LlmxError) as e:
            fn(a, q, k, v, D ** -0.5, algo=bad, **args)
        assert e.value.status == 2
