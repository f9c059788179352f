"""CUDA library vs. the reference's oracle on the golden cases.

Every golden case (the reference's 16-case parity suite,
csrc/test_attention.py:143-201, plus ALiBi / padded / non-causal / decode /
fp32 cases the reference oracle computes) runs through the torch-facing
binding and the C ABI with every kernel family that accepts it, and is
compared (a) with the stored ``ref_attention`` outputs and (b) with the full
fp32 CPU oracle output.  Tolerances: see gpu_helpers.
"""
import numpy as np
import pytest
import torch

import llmx_b200
from cases import make_inputs
from golden_io import load_golden
from gpu_helpers import assert_close, assert_close_np, needs_cuda, oracle_fp32, oracle_padded_fp32

pytestmark = [pytest.mark.gpu, needs_cuda]

CASES = load_golden()
ALGOS = ["simt", "decode", "tcgen05"]


def _run(c, q, k, v, slopes, algo):
    dev = torch.device("cuda", 0)
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    out = torch.full_like(qd, float("nan"))
    kw = dict(alibi_slopes=None if slopes is None else slopes.to(dev), causal=c.causal, algo=algo)
    if c.kind == "padded":
        if c.q_lens:
            kw["q_lens"] = torch.tensor(c.q_lens, dtype=torch.int32, device=dev)
        if c.kv_lens:
            kw["kv_lens"] = torch.tensor(c.kv_lens, dtype=torch.int32, device=dev)
    try:
        llmx_b200.single_mha_attention_half(out, qd, kd, vd, c.sm_scale, c.sliding_window,
                                            c.logits_soft_cap, **kw)
    except llmx_b200.LlmxError as e:
        if e.status == 2:  # LLMX_ERR_UNSUPPORTED: this family does not take the case
            pytest.skip(f"{algo} does not support {c.name}")
        raise
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("case", CASES, ids=[c[0].name for c in CASES])
def test_golden(case, algo):
    c, entry, idx, val = case
    q, k, v, slopes = make_inputs(c)
    out = _run(c, q, k, v, slopes, algo)
    got = out.float().cpu().reshape(-1).numpy()
    dt = q.dtype
    assert_close_np(got[idx], val, dt, f"{c.name}/{algo} vs golden")
    kw = dict(sm_scale=c.sm_scale, logits_soft_cap=c.logits_soft_cap, sliding_window=c.sliding_window,
              alibi=slopes, causal=c.causal)
    if c.kind == "single":
        ref = oracle_fp32(q, k, v, **kw)
    else:
        ref = oracle_padded_fp32(q, k, v, q_lens=c.q_lens, kv_lens=c.kv_lens, **kw)
    assert_close(out, ref, dt, f"{c.name}/{algo} vs oracle")
    llmx_b200.device_status(0)
