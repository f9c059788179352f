"""Multi-GPU partitioning of the attention forward (one process per GPU).

Two ways the work splits across GPUs of one node:

* **batch x head shards** (independent units, no communication): every
  (batch, head) pair is an independent attention problem.  ``shard_units``
  gives each rank a contiguous, balanced slice of the flattened units; each
  rank runs the kernel on its slice.
* **KV split** for long sequences: each rank holds the full query block and a
  share of the keys, computes (O_r, lse_r) over its keys with the kernel
  (``kv_offset`` / ``kv_total`` place the shard's keys at their global
  positions for the causal diagonal and ALiBi), and the partials are merged
  exactly with the log-sum-exp rule

      lse = log sum_r exp(lse_r),   O = sum_r exp(lse_r - lse) O_r

  as NCCL all-reduce MAX of lse_r, a local rescale, and one all-reduce SUM of
  [O_r * w_r | w_r] (w_r = exp(lse_r - max)).  For causal masking each rank
  takes one contiguous key range sized for equal visible work
  (``causal_key_range``: early keys are seen by more queries, so the first
  ranges are shorter); ``zigzag_chunks`` gives the classic two-chunk deal
  (with 2n chunks, rank g takes chunks g and 2n-1-g) for callers that want it.

The reference has no multi-GPU code; its kernel already streams keys through
an online softmax inside one SM (single_mha_kernel.cuh:294-340), and the
merge here is the same running-max / running-sum algebra applied across
shards instead of across blocks (softmax.h:53-110).
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import torch

from . import ops


def shard_units(batch: int, heads: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous range [start, end) of flattened (batch, head) units for `rank`.

    Unit u is (u // heads, u % heads); the ranges differ in size by at most
    one unit and cover every unit exactly once.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    units = batch * heads
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    end = start + base + (1 if rank < extra else 0)
    return start, end


def zigzag_chunks(seq_len: int, world: int, rank: int, align: int = 128) -> List[Tuple[int, int]]:
    """Key ranges [start, end) of `rank` when `seq_len` keys are dealt in
    2 * world chunks, rank g taking chunks g and 2 * world - 1 - g.

    Chunk boundaries are multiples of `align` (the kernel's key block) except
    the last; empty chunks are dropped.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    n = 2 * world
    step = -(-seq_len // n)
    step = -(-step // align) * align
    bounds = [min(seq_len, c * step) for c in range(n + 1)]
    out = []
    for c in sorted({rank, n - 1 - rank}):
        if bounds[c + 1] > bounds[c]:
            out.append((bounds[c], bounds[c + 1]))
    return out


def causal_key_range(seq_len: int, world: int, rank: int, align: int = 16) -> Tuple[int, int]:
    """One contiguous key range [start, end) per rank, sized so that every
    rank has the same number of visible causal (query, key) pairs when all
    `seq_len` queries attend over `seq_len` keys (key j is seen by the
    seq_len - j queries at or below it).

    Every rank holds all queries, so unlike the zig-zag deal one range per
    rank suffices: one kernel launch and one partial per rank.  Range
    boundaries are rounded to multiples of `align`; the ranges cover every
    key exactly once (empty ranges are possible for tiny sequences).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    total = seq_len * (seq_len + 1) / 2
    b = 2 * seq_len + 1

    def bound(r: int) -> int:
        if r <= 0:
            return 0
        if r >= world:
            return seq_len
        # smallest x with x * seq_len - x * (x - 1) / 2 >= r * total / world
        x = (b - math.sqrt(max(0.0, b * b - 8 * r * total / world))) / 2
        return min(seq_len, int(round(x / align)) * align)

    return bound(rank), bound(rank + 1)


def kv_split_ranges(seq_len: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """The key ranges of `rank` for a causal KV split over `world` ranks: one
    contiguous, work-balanced range (``causal_key_range``), so each rank runs
    one launch and holds one partial.

    Measured on B200 (B1 H32 S32768 D128 bf16, causal + ALiBi; slowest rank's
    kernel time as a fraction of a perfect split): 2 ranks 0.96 zig-zag /
    0.92 contiguous, 4 ranks 0.82 / 0.82, 8 ranks 0.71 / 0.79.  At 2 ranks
    the zig-zag deal computes 4% faster, but one partial per rank lets the
    merge gather 16-bit partials instead of all-reducing an fp32 buffer,
    which saves more than that.
    """
    a, b = causal_key_range(seq_len, world, rank)
    return [(a, b)] if b > a else []


def merge_partials(outs: Sequence[torch.Tensor], lses: Sequence[torch.Tensor]):
    """Exact merge of attention partials over disjoint key sets (one rank).

    outs: [B, S, H, D] each (any float type); lses: [B, H, S] fp32 natural-log
    (-inf where a row saw no key).  Returns (O fp32 [B, S, H, D], lse [B, H, S]).
    """
    lse = torch.stack(list(lses), 0)  # [n, B, H, S]
    m = lse.amax(0)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(lse - m_safe)  # exp(-inf) = 0 for empty partials
    wsum = w.sum(0)
    num = None
    for o, wi in zip(outs, w):
        term = o.float() * wi.permute(0, 2, 1).unsqueeze(-1)
        num = term if num is None else num + term
    inv = torch.where(wsum > 0, 1.0 / wsum, torch.zeros_like(wsum))
    out = num * inv.permute(0, 2, 1).unsqueeze(-1)
    lse_out = torch.where(wsum > 0, m_safe + torch.log(wsum), torch.full_like(m, float("-inf")))
    return out, lse_out


def merge_across_ranks(out: torch.Tensor, lse: torch.Tensor, group=None):
    """Exact merge of this rank's partial (out fp32 [B, S, H, D], lse [B, H, S])
    with every other rank's, via all-reduce MAX then one all-reduce SUM.

    Every rank returns the merged (O fp32, lse).  Works on any backend
    torch.distributed supports for these ops (NCCL on GPUs, gloo on CPU).
    """
    import torch.distributed as dist

    m = lse.clone()
    dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(lse - m_safe)  # [B, H, S]; 0 where this rank saw no key
    B, S, H, D = out.shape
    payload = torch.empty(B * S * H * D + B * H * S, dtype=torch.float32, device=out.device)
    num = payload[: B * S * H * D].view(B, S, H, D)
    torch.mul(out.float(), w.permute(0, 2, 1).unsqueeze(-1), out=num)
    payload[B * S * H * D :].copy_(w.reshape(-1))
    dist.all_reduce(payload, op=dist.ReduceOp.SUM, group=group)
    wsum = payload[B * S * H * D :].view(B, H, S)
    inv = torch.where(wsum > 0, 1.0 / wsum, torch.zeros_like(wsum))
    merged = num * inv.permute(0, 2, 1).unsqueeze(-1)
    lse_out = torch.where(wsum > 0, m_safe + torch.log(wsum), torch.full_like(m, float("-inf")))
    return merged, lse_out


def kv_split_attention(
    q: torch.Tensor,
    k_chunks: Sequence[torch.Tensor],
    v_chunks: Sequence[torch.Tensor],
    chunk_offsets: Sequence[int],
    kv_total: int,
    sm_scale: float,
    *,
    alibi_slopes: Optional[torch.Tensor] = None,
    causal: bool = True,
    sliding_window: int = -1,
    group=None,
    out_dtype: Optional[torch.dtype] = None,
):
    """Attention of all of `q` ([B, S, H, D]) over the keys of every rank,
    where this rank holds the key chunks `k_chunks` / `v_chunks`
    ([B, n_c, H_kv, D]) starting at global positions `chunk_offsets`.

    Runs the kernel once per local chunk and merges every chunk of every
    rank of `group` exactly (cross-rank steps skipped when torch.distributed
    is not initialised or the group has one rank) with the library's merge
    kernels.  Returns (O in `out_dtype` (default q's), lse fp32 [B, H, S]) on
    every rank.
    """
    import torch.distributed as dist

    B, S, H, D = q.shape
    outs, lses = [], []
    for kc, vc, off in zip(k_chunks, v_chunks, chunk_offsets):
        o = torch.empty_like(q)
        l = torch.empty(B, H, S, dtype=torch.float32, device=q.device)
        ops.single_mha_attention_half(o, q, kc, vc, sm_scale, sliding_window, alibi_slopes=alibi_slopes,
                                      causal=causal, lse=l, kv_offset=int(off), kv_total=int(kv_total))
        outs.append(o)
        lses.append(l)
    multi = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
    return _merge_cuda(outs, lses, q, multi, group, out_dtype)


def _merge_cuda(outs, lses, q, multi, group, out_dtype):
    """The merge on the GPU: row max of lse over every shard (all-reduce MAX),
    one scale kernel writing [num | wsum] for the local partials, one
    all-reduce SUM of that buffer, one finish kernel.  With one partial per
    rank and at most three ranks the partials are all-gathered instead and
    merged locally (no MAX / SUM all-reduce)."""
    import ctypes

    import torch.distributed as dist

    from . import _lib

    B, S, H, D = q.shape
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("the KV-split merge takes fp16 or bf16 partials")
    world = dist.get_world_size(group) if multi else 1
    if multi and world <= 3 and len(outs) == 1:
        # One partial per rank and few ranks: gathering every rank's 16-bit O
        # and fp32 lse moves (world - 1) x (2 D + 4) bytes per row into each
        # rank, against 2 (world - 1) / world x (4 D + 4) for the all-reduce
        # of the fp32 [num | wsum] buffer; the merge then runs locally over
        # all partials, in the same fp32 arithmetic.
        o_all = torch.empty((world,) + tuple(q.shape), dtype=q.dtype, device=q.device)
        l_all = torch.empty((world, B, H, S), dtype=torch.float32, device=q.device)
        dist.all_gather_into_tensor(o_all, outs[0].contiguous(), group=group)
        dist.all_gather_into_tensor(l_all, lses[0].contiguous(), group=group)
        outs, lses, multi = list(o_all.unbind(0)), list(l_all.unbind(0)), False
    if lses:
        m = torch.stack(list(lses), 0).amax(0)
    else:
        m = torch.full((B, H, S), float("-inf"), device=q.device)
    if multi:
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    n = B * S * H * D
    payload = torch.empty(n + B * H * S, dtype=torch.float32, device=q.device)
    num, wsum = payload[:n], payload[n:]
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    dt = _lib.DTYPE["bf16" if q.dtype == torch.bfloat16 else "fp16"]
    outs = [o.contiguous() for o in outs]
    optrs = (ctypes.c_void_p * max(1, len(outs)))(*[o.data_ptr() for o in outs])
    lptrs = (ctypes.c_void_p * max(1, len(lses)))(*[l.data_ptr() for l in lses])
    _lib.check(lib.llmx_attn_lse_merge_scale(len(outs), optrs, lptrs, m.data_ptr(), dt, B, S, H, D,
                                             num.data_ptr(), wsum.data_ptr(), stream))
    if multi:
        dist.all_reduce(payload, op=dist.ReduceOp.SUM, group=group)
    out = torch.empty(B, S, H, D, dtype=out_dtype or q.dtype, device=q.device)
    if out.dtype != q.dtype:
        tmp = torch.empty_like(q)
    else:
        tmp = out
    lse = torch.empty(B, H, S, dtype=torch.float32, device=q.device)
    _lib.check(lib.llmx_attn_lse_merge_finish(num.data_ptr(), wsum.data_ptr(), m.data_ptr(), dt, B, S, H, D,
                                              tmp.data_ptr(), lse.data_ptr(), stream))
    if tmp is not out:
        out.copy_(tmp)
    return out, lse
