"""Edge cases through the C ABI and the torch binding, every kernel family.

Empty and ragged sequences, lengths past the padded extent (clamped), rows
that see no key, non-contiguous K/V views, odd head dims, GQA groups that do
not divide the CTA slice, the log-sum-exp output, and a non-default stream.
Tolerances: see gpu_helpers.
"""
import pytest
import torch

import llmx_b200
import oracle
from gpu_helpers import assert_close, needs_cuda

pytestmark = [pytest.mark.gpu, needs_cuda]

DEV = "cuda"


def rand(*shape, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).to(DEV)


def call(q, k, v, algo="auto", **kw):
    out = torch.full_like(q, float("nan"))
    try:
        llmx_b200.single_mha_attention_half(out, q, k, v, q.shape[-1] ** -0.5, algo=algo, **kw)
    except llmx_b200.LlmxError as e:
        if e.status == 2 and algo != "auto":
            pytest.skip(f"{algo} does not take this case")
        raise
    torch.cuda.synchronize()
    return out


def ref_padded(q, k, v, q_lens, kv_lens, **kw):
    return oracle.attention_ref_padded(q.float().cpu(), k.float().cpu(), v.float().cpu(), q_lens=q_lens,
                                       kv_lens=kv_lens, return_lse=True, **kw)


ALGOS = ["auto", "simt", "decode", "tcgen05"]


@pytest.mark.parametrize("algo", ALGOS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ragged_batch_with_empty_sequences(algo, dtype):
    B, S, H, Hkv, D = 5, 200, 4, 2, 128
    q, k, v = rand(B, S, H, D, dtype=dtype), rand(B, S, Hkv, D, dtype=dtype, seed=1), rand(B, S, Hkv, D, dtype=dtype, seed=2)
    q_lens = [0, 1, 77, 200, 129]
    kv_lens = [5, 0, 131, 200, 129]
    ql = torch.tensor(q_lens, dtype=torch.int32, device=DEV)
    kl = torch.tensor(kv_lens, dtype=torch.int32, device=DEV)
    lse = torch.empty(B, H, S, device=DEV)
    out = call(q, k, v, algo, q_lens=ql, kv_lens=kl, lse=lse, causal=False)
    ref, ref_lse = ref_padded(q, k, v, q_lens, kv_lens, causal=False)
    assert_close(out, ref, dtype, f"ragged/{algo}")
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    torch.testing.assert_close(lse.cpu()[fin], ref_lse[fin], atol=2e-3, rtol=0)


@pytest.mark.parametrize("algo", ALGOS)
def test_lengths_past_extent_are_clamped(algo):
    B, S, H, D = 2, 64, 2, 64
    q, k, v = rand(B, S, H, D), rand(B, S, H, D, seed=1), rand(B, S, H, D, seed=2)
    big = torch.tensor([10**6, 64], dtype=torch.int32, device=DEV)
    out = call(q, k, v, algo, q_lens=big, kv_lens=big)
    ref, _ = ref_padded(q, k, v, [64, 64], [64, 64])
    assert_close(out, ref, torch.bfloat16, f"clamp/{algo}")


@pytest.mark.parametrize("algo", ["simt", "tcgen05"])
def test_causal_rows_without_keys_are_zero(algo):
    # kv_len < q_len: the first q_len - kv_len rows see no key (reference: NaN)
    q, k, v = rand(96, 2, 128), rand(40, 2, 128, seed=1), rand(40, 2, 128, seed=2)
    out = call(q, k, v, algo)
    ref = oracle.attention_ref(q.float().cpu(), k.float().cpu(), v.float().cpu())
    assert torch.all(out[:56] == 0)
    assert_close(out, ref, torch.bfloat16, "kv<q")


@pytest.mark.parametrize("algo", ["auto", "simt", "tcgen05", "decode"])
def test_non_contiguous_kv_views(algo):
    # K and V as views of a packed [B, S, 3, H, D] projection
    B, S, H, D = 2, 130, 4, 128
    qkv = rand(B, S, 3, H, D)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    if algo == "decode":
        q = q[:, :1]
    out = call(q, k, v, algo, causal=True)
    ref, _ = ref_padded(q, k, v, None, None, causal=True)
    assert_close(out, ref, torch.bfloat16, f"views/{algo}")


@pytest.mark.parametrize("D", [32, 80, 96, 256])
def test_other_head_dims(D):
    q, k, v = rand(70, 3, D), rand(90, 1, D, seed=1), rand(90, 1, D, seed=2)
    out = call(q, k, v, "auto", logits_soft_cap=20.0, sliding_window=33)
    ref = oracle.attention_ref(q.float().cpu(), k.float().cpu(), v.float().cpu(), logits_soft_cap=20.0,
                               sliding_window=33)
    assert_close(out, ref, torch.bfloat16, f"D={D}")


@pytest.mark.parametrize("group", [1, 3, 6, 12])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_decode_gqa_groups(group, D):
    B, Hkv, S = 3, 2, 700
    H = Hkv * group
    q, k, v = rand(B, 1, H, D), rand(B, S, Hkv, D, seed=1), rand(B, S, Hkv, D, seed=2)
    kv_lens = [700, 1, 333]
    kl = torch.tensor(kv_lens, dtype=torch.int32, device=DEV)
    a = oracle.alibi_slopes(H).to(DEV)
    out = call(q, k, v, "decode", kv_lens=kl, alibi_slopes=a, sliding_window=300)
    ref, _ = ref_padded(q, k, v, [1] * B, kv_lens, alibi=a.cpu(), sliding_window=300)
    assert_close(out, ref, torch.bfloat16, f"decode G={group} D={D}")


def test_non_default_stream():
    q, k, v = rand(256, 4, 128), rand(256, 4, 128, seed=1), rand(256, 4, 128, seed=2)
    s = torch.cuda.Stream()
    out = torch.empty_like(q)
    with torch.cuda.stream(s):
        llmx_b200.single_mha_attention_half(out, q, k, v, 128 ** -0.5)
    s.synchronize()
    ref = oracle.attention_ref(q.float().cpu(), k.float().cpu(), v.float().cpu())
    assert_close(out, ref, torch.bfloat16, "stream")


def test_reference_signature_checks():
    q = rand(8, 4, 64)
    with pytest.raises(RuntimeError):
        llmx_b200.single_mha_attention_half(torch.empty_like(q), q, rand(8, 3, 64), rand(8, 3, 64), 0.125)
    with pytest.raises(RuntimeError):
        llmx_b200.single_mha_attention_half(torch.empty_like(q), q, rand(8, 4, 32), rand(8, 4, 32), 0.125)
    with pytest.raises(RuntimeError):
        llmx_b200.single_mha_attention_half(torch.empty_like(q), q.cpu(), q.cpu(), q.cpu(), 0.125)
    llmx_b200.device_status(0)


def test_non_positive_scale_leaves_the_tensor_core_kernel():
    # The tensor-core softmax takes its row max on raw scores, which needs
    # sm_scale > 0; other scales are routed to the SIMT kernel (auto) or
    # refused (forced), and still match the oracle.
    q, k, v = rand(1, 200, 2, 64), rand(1, 200, 2, 64, seed=1), rand(1, 200, 2, 64, seed=2)
    for scale in (-0.125, 0.0):
        out = torch.empty_like(q)
        assert llmx_b200.selected_algo(out, q, k, v, scale) == "simt"
        llmx_b200.single_mha_attention_half(out, q, k, v, scale)
        torch.cuda.synchronize()
        ref = oracle.attention_ref(q[0].float().cpu(), k[0].float().cpu(), v[0].float().cpu(), sm_scale=scale)
        assert_close(out[0], ref, torch.bfloat16, f"scale {scale}")
        with pytest.raises(llmx_b200.LlmxError):
            llmx_b200.single_mha_attention_half(out, q, k, v, scale, algo="tcgen05")
