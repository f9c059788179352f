"""llmx_attn_decode_noalloc: split-KV decode without any allocation.

Serving engines that reserve all device memory at start-up, and latency-
critical loops that cannot afford cudaMalloc's device-wide synchronisation,
cannot hand the library a workspace.  This entry point keeps the split
partials in a static device array instead.  The test calls it through the C
ABI, twice in a row on different inputs (the array keeps the previous call's
contents), and checks each result against llmx_attn_fwd given a workspace
and against the fp32 CPU oracle directly, within the GPU tests' tolerance
(gpu_helpers).  It also checks that a request
larger than the array is refused before anything is launched.

This file is collected last so that a failing run has already run every
other test.
"""
import ctypes

import pytest
import torch

import oracle
from gpu_helpers import assert_close, needs_cuda
from llmx_b200 import _lib, ops

pytestmark = [pytest.mark.gpu, needs_cuda]


def _inputs(seed, B=16, H=32, Hkv=8, S=3000, D=128):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, S + 1, (B,), generator=g)
    q = torch.randn(B, 1, H, D, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    slopes = torch.pow(2.0, -8.0 * torch.arange(1, H + 1) / H).float().cuda()
    return q, k, v, lens.to(torch.int32).cuda(), slopes


def _noalloc(q, k, v, lens, slopes):
    out = torch.full_like(q, float("nan"))
    p, keep = ops.build_params(out, q, k, v, q.shape[-1] ** -0.5, alibi_slopes=slopes, kv_lens=lens,
                               algo="decode")
    st = _lib.load().llmx_attn_decode_noalloc(ctypes.byref(p),
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st)
    return out


def test_noalloc_decode_matches_workspace_decode_twice():
    for seed in (0, 1):
        q, k, v, lens, slopes = _inputs(seed)
        ref = torch.empty_like(q)
        ops.single_mha_attention_half(ref, q, k, v, q.shape[-1] ** -0.5, alibi_slopes=slopes, kv_lens=lens,
                                      algo="decode")
        out = _noalloc(q, k, v, lens, slopes)
        torch.cuda.synchronize()
        assert_close(out, ref, torch.bfloat16, f"no-alloc decode, call {seed + 1}")
        direct = oracle.attention_ref_padded(q.float().cpu(), k.float().cpu(), v.float().cpu(),
                                             kv_lens=lens.cpu().tolist(), alibi=slopes.cpu(),
                                             sm_scale=q.shape[-1] ** -0.5)
        assert_close(out, direct, torch.bfloat16, f"no-alloc decode vs the oracle, call {seed + 1}")
    ops.device_status(0)


def test_noalloc_refuses_requests_larger_than_the_array():
    lib = _lib.load()
    p = _lib.AttnParams()
    lib.llmx_attn_params_init(ctypes.byref(p))
    p.dtype, p.batch, p.n_heads, p.n_kv_heads, p.head_dim = 2, 512, 64, 64, 256
    p.max_q_len, p.max_kv_len = 1, 65536
    # addresses are never dereferenced: the request is refused before any launch
    p.q, p.k, p.v, p.o = 0x100000, 0x200000, 0x300000, 0x400000
    p.sm_scale = 0.0625
    lib.llmx_attn_set_contiguous_strides(ctypes.byref(p))
    st = lib.llmx_attn_decode_noalloc(ctypes.byref(p), None)
    assert _lib.STATUS_NAMES[st] == "LLMX_ERR_WORKSPACE_TOO_SMALL"
    assert b"static array" in lib.llmx_attn_last_error()
