"""The CPU oracle against the reference's own oracle (golden fixtures).

The fixtures hold ``ref_attention`` (csrc/test_attention.py:41-93) outputs on
seeded CPU inputs; this pins ``oracle.attention_ref`` before any kernel is
compared with it.  The oracle computes in fp32 with a different reduction
order, so 16-bit outputs may differ by one unit in the last place after the
final cast; fp32 outputs agree to 2e-6.
"""
import numpy as np
import pytest
import torch

import oracle
from cases import make_inputs
from golden_io import load_golden, to_numpy, ulp_tol

CASES = load_golden()


def run_oracle(c, q, k, v, slopes):
    kw = dict(sm_scale=c.sm_scale, logits_soft_cap=c.logits_soft_cap,
              sliding_window=c.sliding_window, alibi=slopes, causal=c.causal)
    if c.kind == "single":
        return oracle.attention_ref(q, k, v, **kw)
    return oracle.attention_ref_padded(q, k, v, q_lens=c.q_lens, kv_lens=c.kv_lens, **kw)


@pytest.mark.parametrize("case", CASES, ids=[c[0].name for c in CASES])
def test_oracle_matches_reference_oracle(case):
    c, entry, idx, val = case
    q, k, v, slopes = make_inputs(c)
    sums = [float(t.double().sum()) for t in (q, k, v)]
    assert np.allclose(sums, entry["input_checksums"], rtol=0, atol=1e-6), \
        "seeded inputs differ from the ones the fixtures were made from"
    out = to_numpy(run_oracle(c, q, k, v, slopes))
    got = out[idx]
    tol = 2e-6 if c.dtype == "fp32" else ulp_tol(c.dtype, val)
    assert np.all(np.abs(got - val) <= tol), float(np.max(np.abs(got - val)))
    assert abs(out.astype(np.float64).sum() - entry["out_sum"]) <= 1e-3 * max(1.0, entry["out_abs_sum"]) ** 0.5


def test_oracle_lse_consistent():
    """lse from the oracle reproduces softmax: sum_j exp(s_j - lse) == 1."""
    g = torch.Generator().manual_seed(5)
    q = torch.randn(9, 2, 16, generator=g)
    k = torch.randn(13, 2, 16, generator=g)
    v = torch.eye(16)[:13].view(13, 1, 16).expand(13, 2, 16).contiguous()
    o, lse = oracle.attention_ref(q, k, v, return_lse=True, causal=False)
    # with V = identity rows, O[i, h, j] = softmax weight of key j
    w = o[:, :, :13].sum(-1)
    assert torch.allclose(w, torch.ones_like(w), atol=1e-5)
    s = torch.einsum("qhd,khd->hqk", q, k) / 4.0
    ref_lse = torch.logsumexp(s, dim=-1)
    assert torch.allclose(lse, ref_lse, atol=1e-5)


def test_oracle_empty_rows_are_zero():
    q = torch.randn(4, 1, 8)
    k = torch.randn(2, 1, 8)
    v = torch.randn(2, 1, 8)
    # causal with kv_len < q_len: rows 0 and 1 see no key
    o, lse = oracle.attention_ref(q, k, v, return_lse=True, causal=True)
    assert torch.all(o[:2] == 0) and torch.all(torch.isinf(lse[0, :2]))
    assert torch.all(torch.isfinite(lse[0, 2:]))
