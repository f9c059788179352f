"""head_dim 256 on the tensor-core prefill kernel (one 128-row query tile per
work item, double-buffered scores), against the CPU oracle.

Covers causal / non-causal, ALiBi (folded into QK^T), soft-cap, sliding
window, GQA, padded batches, key shards (kv_offset / kv_total), the lse
output, items of 1, 2 and more key blocks (the QK^T-ahead pipeline's edge
cases), fp16 and bf16, and that the queued (workspace) and one-CTA-per-item
launches agree bit for bit.  Tolerances: see gpu_helpers.
"""
import ctypes

import pytest
import torch

import llmx_b200
import oracle
from gpu_helpers import assert_close, needs_cuda
from llmx_b200 import _lib, ops

pytestmark = [pytest.mark.gpu, needs_cuda]

D = 256


def rand(*shape, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).cuda()


def run(q, k, v, **kw):
    out = torch.full_like(q, float("nan"))
    assert llmx_b200.selected_algo(out, q, k, v, D ** -0.5, **{x: y for x, y in kw.items() if x != "lse"}) == "tcgen05"
    llmx_b200.single_mha_attention_half(out, q, k, v, D ** -0.5, **kw)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("S", [100, 128, 200, 256, 600])  # 1, 1, 2, 2, 5 key blocks for the last tile
@pytest.mark.parametrize("causal", [True, False])
def test_shapes_and_block_counts(dtype, S, causal):
    H = 2
    q, k, v = rand(1, S, H, D, dtype=dtype), rand(1, S, H, D, dtype=dtype, seed=1), rand(1, S, H, D, dtype=dtype, seed=2)
    lse = torch.empty(1, H, S, device="cuda")
    out = run(q, k, v, causal=causal, lse=lse)
    ref, lref = oracle.attention_ref(q[0].float().cpu(), k[0].float().cpu(), v[0].float().cpu(), causal=causal,
                                     return_lse=True)
    assert_close(out[0], ref, dtype, f"S={S} causal={causal}")
    torch.testing.assert_close(lse[0].cpu(), lref, atol=2e-3, rtol=0)


@pytest.mark.parametrize("features", ["alibi", "softcap", "alibi_softcap", "window"])
def test_score_features(features):
    S, H = 700, 4
    q, k, v = rand(1, S, H, D), rand(1, S, H, D, seed=1), rand(1, S, H, D, seed=2)
    kw, rkw = {}, {}
    if "alibi" in features:
        slopes = oracle.alibi_slopes(H)
        kw["alibi_slopes"], rkw["alibi"] = slopes.cuda(), slopes
    if "softcap" in features:
        kw["logits_soft_cap"] = rkw["logits_soft_cap"] = 30.0
    if features == "window":
        kw["sliding_window"] = rkw["sliding_window"] = 200
    out = run(q, k, v, **kw)
    ref = oracle.attention_ref(q[0].float().cpu(), k[0].float().cpu(), v[0].float().cpu(), **rkw)
    assert_close(out[0], ref, torch.bfloat16, features)


def test_gqa_and_padded_batch():
    B, S, H, Hkv = 3, 520, 8, 2
    q, k, v = rand(B, S, H, D), rand(B, S, Hkv, D, seed=1), rand(B, S, Hkv, D, seed=2)
    lens = [520, 131, 300]
    ql = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = run(q, k, v, q_lens=ql, kv_lens=ql)
    ref = oracle.attention_ref_padded(q.float().cpu(), k.float().cpu(), v.float().cpu(), q_lens=lens, kv_lens=lens)
    for b, n in enumerate(lens):
        assert_close(out[b, :n], ref[b, :n], torch.bfloat16, f"b={b}")
        assert torch.all(out[b, n:] == 0)


def test_key_shard():
    S, H = 900, 2
    a0, a1 = 256, 640
    q, k, v = rand(1, S, H, D), rand(1, S, H, D, seed=1), rand(1, S, H, D, seed=2)
    slopes = oracle.alibi_slopes(H)
    lse = torch.empty(1, H, S, device="cuda")
    out = run(q, k[:, a0:a1].contiguous(), v[:, a0:a1].contiguous(), alibi_slopes=slopes.cuda(), lse=lse,
              kv_offset=a0, kv_total=S)
    ref, lref = oracle.attention_ref(q[0].float().cpu(), k[0, a0:a1].float().cpu(), v[0, a0:a1].float().cpu(),
                                     alibi=slopes, return_lse=True, kv_offset=a0, kv_total=S)
    assert_close(out[0], ref, torch.bfloat16, "shard")
    fin = torch.isfinite(lref)
    assert torch.equal(torch.isfinite(lse[0].cpu()), fin)
    torch.testing.assert_close(lse[0].cpu()[fin], lref[fin], atol=2e-3, rtol=0)


def test_queued_and_per_item_launches_agree():
    B, S, H = 2, 2048, 8  # 256 items: more than one per SM
    q, k, v = rand(B, S, H, D), rand(B, S, H, D, seed=1), rand(B, S, H, D, seed=2)
    queued = run(q, k, v)
    per_item = torch.empty_like(q)
    p, keep = ops.build_params(per_item, q, k, v, D ** -0.5, algo="tcgen05")
    _lib.check(_lib.load().llmx_attn_fwd(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert torch.equal(queued, per_item)
    # the pipeline's barrier phases under different timings: repeated runs are bit-identical
    for _ in range(6):
        assert torch.equal(run(q, k, v), queued)
    rows = slice(S - 128, S)
    ref = oracle.attention_ref(q[1, rows].float().cpu(), k[1].float().cpu(), v[1].float().cpu())
    assert_close(queued[1, rows], ref, torch.bfloat16, "last rows")
