"""The torch binding (llmx_b200/csrc/llmx_bind.cpp, module llmx_b200.llmx_bind)
and the reference's own boundary sources, without a GPU.

* the binding builds as a torch extension over libllmx_attn.so, imports, and
  exposes single_mha_attention_half with the reference's argument names,
  order and defaults (csrc/llmx_bind.cpp:72-77) plus the keyword extensions;
* the reference's csrc/llmx_bind.cpp and test/cuda/mha_attention_test.cpp
  compile unchanged against include/ (skipped where the reference source is
  not present; oracle/build_ref_boundary.py is the recipe).
"""
import importlib

import pytest


def test_binding_builds_and_exposes_the_reference_signature():
    from llmx_b200 import build as b

    b.build_binding()
    m = importlib.import_module("llmx_b200.llmx_bind")
    assert m.abi_version() == 3
    doc = m.single_mha_attention_half.__doc__
    # positional part identical to the reference's, then the keyword-only extensions
    sig = doc.splitlines()[0]
    names = [p.split(":")[0].strip() for p in sig[sig.index("(") + 1:sig.rindex(")")].split(",")]
    assert names == ["output", "q", "k", "v", "sm_scale", "sliding_window", "logits_soft_cap", "*", "alibi_slopes",
                     "causal", "q_lens", "kv_lens", "lse", "algo", "kv_offset", "kv_total"], sig
    for piece in ("sliding_window: typing.SupportsInt = -1", "logits_soft_cap: typing.SupportsFloat = 0.0",
                  "causal: bool = True"):
        assert piece.split(":")[0] in sig and piece.split("= ")[-1] in sig


def test_binding_rejects_cpu_tensors_like_the_reference():
    import torch

    m = importlib.import_module("llmx_b200.llmx_bind")
    q = torch.zeros(4, 2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        m.single_mha_attention_half(torch.empty_like(q), q, q, q, 0.125)
    with pytest.raises(RuntimeError, match="same dtype"):
        m.single_mha_attention_half(torch.empty_like(q), q, q.bfloat16(), q, 0.125)
    with pytest.raises(RuntimeError, match="3-D"):
        m.single_mha_attention_half(torch.empty_like(q), q[0], q, q, 0.125)


def test_reference_boundary_sources_compile_unchanged():
    from oracle import build_ref_boundary as rb

    if rb.reference_root() is None:
        pytest.skip("reference source not present")
    rb.build(syntax_only=True)
