"""Host-resident inputs (llmx_b200.HostAttention / attention_from_host):
the chunked upload / kernel / download pipeline gives exactly the result of
the device call on the same data, with and without the causal row pieces of
the last batch element, and matches the fp32 oracle."""
import pytest
import torch

import llmx_b200
import oracle
from gpu_helpers import assert_close, needs_cuda

pytestmark = [pytest.mark.gpu, needs_cuda]


def _host(*shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).pin_memory()


@pytest.mark.parametrize("B,S,H,D,causal,alibi,chunks,tail", [
    (3, 1024, 4, 128, True, False, 2, 4),    # last element in four row pieces
    (3, 1024, 4, 128, True, True, 3, 3),     # ALiBi (keys last to first), pieces of 384 rows
    (2, 512, 4, 64, True, False, 2, 1),      # no row pieces
    (2, 512, 4, 64, False, True, 2, 4),      # non-causal: no row pieces
    (1, 2048, 8, 128, True, False, 1, 4),    # one element, all of it in row pieces
])
def test_host_pipeline_equals_device_call(B, S, H, D, causal, alibi, chunks, tail):
    dtype = torch.bfloat16
    qh, kh, vh = (_host(B, S, H, D, dtype=dtype, seed=s) for s in range(3))
    oh = torch.full_like(qh, float("nan")).pin_memory()
    slopes = oracle.alibi_slopes(H).cuda() if alibi else None
    run = llmx_b200.HostAttention(qh, kh, "cuda", chunks=chunks, tail_pieces=tail)
    for _ in range(2):  # buffers and streams reused by a second call
        run(oh, qh, kh, vh, D ** -0.5, causal=causal, alibi_slopes=slopes)
        torch.cuda.current_stream().synchronize()
    ref = torch.empty(B, S, H, D, dtype=dtype, device="cuda")
    llmx_b200.single_mha_attention_half(ref, qh.cuda(), kh.cuda(), vh.cuda(), D ** -0.5, causal=causal,
                                        alibi_slopes=slopes)
    torch.cuda.synchronize()
    assert torch.equal(oh, ref.cpu())


def test_attention_from_host_padded_batch_against_oracle():
    B, S, H, D = 3, 384, 4, 64
    dtype = torch.float16
    qh, kh, vh = (_host(B, S, H, D, dtype=dtype, seed=10 + s) for s in range(3))
    oh = torch.empty_like(qh).pin_memory()
    lens = torch.tensor([384, 200, 317], dtype=torch.int32)
    llmx_b200.attention_from_host(oh, qh, kh, vh, D ** -0.5, chunks=3, causal=True, q_lens=lens.cuda(),
                                  kv_lens=lens.cuda())
    for b in range(B):
        n = int(lens[b])
        ref = oracle.attention_ref(qh[b, :n].float(), kh[b, :n].float(), vh[b, :n].float(), sm_scale=D ** -0.5, causal=True)
        assert_close(oh[b, :n], ref, dtype, f"padded batch {b}")
        assert torch.count_nonzero(oh[b, n:]) == 0  # padded query rows are written as zeros


def test_host_pipeline_needs_pinned_memory():
    q = torch.randn(1, 256, 2, 64, dtype=torch.bfloat16)
    run = llmx_b200.HostAttention(q, q, "cuda", chunks=1)
    with pytest.raises(RuntimeError, match="pinned"):
        run(torch.empty_like(q), q, q, q, 0.125)
