"""CPU oracle for llmx's attention forward path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker (or as the timed CPU stand-in for the
reference's CPU path).  The product path (``llmx_b200`` and its CUDA library)
never calls it.

The arithmetic restates the reference's fp32 oracle ``ref_attention``
(``csrc/test_attention.py:41-93``) and the kernel semantics it is pinned
against:

* scores = (q . k) * sm_scale, computed in fp32        (test_attention.py:55-69)
* optional logits soft-cap: tanh(s / cap) * cap        (test_attention.py:71-72;
  kernel form params.h:35-50)
* optional ALiBi: + slope[h] * j, j = absolute key index (test_attention.py:73-77;
  kernel mask.h:33-36,75-77)
* causal mask aligned bottom-right: key j visible to query i iff
  j <= i + (kv_len - q_len)                             (test_attention.py:79-85;
  kernel mask.h:54-63)
* sliding window: masked iff (i + kv_len - q_len) - j > window
                                                        (test_attention.py:82-83; mask.h:60,66)
* GQA: query head h reads kv head h // group           (test_attention.py:61-64;
  single_mha_kernel.cuh:434-441)
* softmax over keys in fp32, O = P V, one final cast to the input dtype
                                                        (test_attention.py:89-93)

Extensions beyond the reference signature (the same arithmetic, applied to
more inputs): a ``causal=False`` mode, per-sequence query/key lengths for
padded batches, a caller-supplied ``sm_scale`` (the kernel API takes one,
``attention_api.h:8-14``; the reference oracle hard-codes 1/sqrt(D)), the
per-row log-sum-exp used by split-KV merging, and key slices (``kv_offset``
/ ``kv_total``: the same mask and ALiBi evaluated at the keys' global
positions).  A row that sees no key at all
(an empty sequence, or causal with kv_len < q_len) yields O = 0 and
lse = -inf; the reference never produces such a row (it asserts
kv_len >= q_len, test_attention.py:51).
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

__all__ = [
    "alibi_slopes",
    "attention_ref",
    "attention_ref_chunked",
    "attention_ref_padded",
]


def alibi_slopes(n_heads: int) -> torch.Tensor:
    """ALiBi slopes m_h = 2^(-8(h+1)/H), fp32, as every workload here defines them."""
    h = torch.arange(n_heads, dtype=torch.float64)
    return torch.pow(2.0, -8.0 * (h + 1.0) / n_heads).to(torch.float32)


def _visible_mask(q_len: int, kv_len: int, causal: bool, sliding_window: int, kv_offset: int = 0,
                  kv_total: Optional[int] = None) -> torch.Tensor:
    """Boolean [q_len, kv_len] mask of the keys each query row may attend to.

    Bottom-right aligned causal mask and sliding window, restating
    ``mask.h:54-66`` / ``test_attention.py:79-85`` with explicit index compares.
    For a slice of a sequence's keys, local key j sits at global position
    kv_offset + j and the diagonal uses the full key length kv_total.
    """
    kfull = kv_len if kv_total is None else kv_total
    i = torch.arange(q_len).view(q_len, 1)
    j = torch.arange(kv_len).view(1, kv_len) + kv_offset
    diag = i + (kfull - q_len)  # query row i on the key axis
    vis = torch.ones(q_len, kv_len, dtype=torch.bool)
    if causal:
        vis &= j <= diag
    if sliding_window >= 0:
        vis &= (diag - j) <= sliding_window
    return vis


def attention_ref(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    sm_scale: Optional[float] = None,
    logits_soft_cap: float = 0.0,
    sliding_window: int = -1,
    alibi: Optional[torch.Tensor] = None,
    causal: bool = True,
    return_lse: bool = False,
    compute_dtype: torch.dtype = torch.float32,
    kv_offset: int = 0,
    kv_total: Optional[int] = None,
):
    """One sequence of attention on CPU.

    q: [q_len, n_heads, D]; k, v: [kv_len, n_kv_heads, D] (any float dtype).
    Returns O [q_len, n_heads, D] in q's dtype (and lse [n_heads, q_len] fp32,
    natural log, when ``return_lse``).  Follows ``ref_attention``
    (csrc/test_attention.py:41-93); see the module docstring for the rules.
    """
    q_len, n_heads, d = q.shape
    kv_len, n_kv_heads, _ = k.shape
    out_dtype = q.dtype
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(d)
    if n_heads % n_kv_heads != 0:
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    group = n_heads // n_kv_heads

    qf = q.to(compute_dtype).permute(1, 0, 2)  # [H, q, D]
    kf = k.to(compute_dtype).permute(1, 0, 2)  # [Hkv, kv, D]
    vf = v.to(compute_dtype).permute(1, 0, 2)
    if group > 1:
        kf = kf.repeat_interleave(group, dim=0)
        vf = vf.repeat_interleave(group, dim=0)

    s = torch.matmul(qf, kf.transpose(1, 2)) * sm_scale  # [H, q, kv]
    if logits_soft_cap != 0.0:
        s = torch.tanh(s / logits_soft_cap) * logits_soft_cap
    if alibi is not None:
        j = torch.arange(kv_len, dtype=compute_dtype) + kv_offset
        s = s + alibi.to(compute_dtype).view(n_heads, 1, 1) * j.view(1, 1, kv_len)

    vis = _visible_mask(q_len, kv_len, causal, sliding_window, kv_offset, kv_total)
    s = s.masked_fill(~vis.unsqueeze(0), float("-inf"))

    row_any = vis.any(dim=1)  # [q]
    m = s.amax(dim=-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m)
    l = p.sum(dim=-1, keepdim=True)
    l_safe = torch.where(l > 0, l, torch.ones_like(l))
    o = torch.matmul(p / l_safe, vf)  # [H, q, D]
    o = o * row_any.view(1, q_len, 1).to(o.dtype)
    out = o.permute(1, 0, 2).contiguous().to(out_dtype)
    if not return_lse:
        return out
    lse = (m + torch.log(l_safe)).squeeze(-1)
    lse = torch.where(row_any.view(1, q_len), lse, torch.full_like(lse, float("-inf")))
    return out, lse.to(torch.float32)


def attention_ref_padded(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    q_lens: Optional[Sequence[int]] = None,
    kv_lens: Optional[Sequence[int]] = None,
    units: Optional[Sequence[tuple]] = None,
    return_lse: bool = False,
    **kw,
):
    """Batched, padded attention: q [B, Sq, H, D], k/v [B, Skv, Hkv, D].

    Sequence b uses its first q_lens[b] query rows and kv_lens[b] keys; padded
    query rows come back as 0 (lse -inf).  ``units`` optionally restricts the
    work to a list of (b, h) pairs (the rest of O stays 0), so that large
    workloads can be checked on a seeded subset.  Each sequence is one
    ``attention_ref`` call, as the reference runs one sequence per call
    (attention_api.cpp:41, batch_size = 1).
    """
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    group = H // Hkv
    q_lens = [Sq] * B if q_lens is None else [int(x) for x in q_lens]
    kv_lens = [Skv] * B if kv_lens is None else [int(x) for x in kv_lens]
    out = torch.zeros_like(q)
    lse = torch.full((B, H, Sq), float("-inf"), dtype=torch.float32)
    alibi = kw.pop("alibi", None)
    by_batch = {}
    if units is None:
        for b in range(B):
            by_batch[b] = list(range(H))
    else:
        for b, h in units:
            by_batch.setdefault(int(b), []).append(int(h))
    for b, heads in by_batch.items():
        ql, kl = q_lens[b], kv_lens[b]
        if ql == 0 or kl == 0:
            continue
        for h in sorted(set(heads)):
            kvh = h // group
            a = None if alibi is None else alibi[h : h + 1]
            o_bh, l_bh = attention_ref(
                q[b, :ql, h : h + 1],
                k[b, :kl, kvh : kvh + 1],
                v[b, :kl, kvh : kvh + 1],
                alibi=a,
                return_lse=True,
                **kw,
            )
            out[b, :ql, h] = o_bh[:, 0]
            lse[b, h, :ql] = l_bh[0]
    return (out, lse) if return_lse else out


def attention_ref_chunked(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    sm_scale: Optional[float] = None,
    alibi: Optional[torch.Tensor] = None,
    causal: bool = True,
    rows: Optional[tuple] = None,
    heads: Optional[Sequence[int]] = None,
    max_elems: int = 1 << 28,
):
    """Whole-batch fp32 oracle on whatever device q lives on, in query-row
    blocks, so that full-size workloads (e.g. 32768 x 32768 scores per head)
    can be checked completely on a GPU.

    q: [B, Sq, H, D]; k, v: [B, Skv, Hkv, D] (all rows valid, no padding).
    The arithmetic is ``attention_ref``'s (fp32 scores, ALiBi + slope * j,
    bottom-right causal mask, softmax, P V) evaluated on row blocks of at most
    ``max_elems`` scores.  ``rows`` = (r0, r1) restricts the query rows and
    ``heads`` the heads.  Returns (O fp32 [B, r1 - r0, len(heads), D],
    lse fp32 [B, len(heads), r1 - r0]).
    """
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    group = H // Hkv
    dev = q.device
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    r0, r1 = (0, Sq) if rows is None else rows
    heads = list(range(H)) if heads is None else list(heads)
    out = torch.empty(B, r1 - r0, len(heads), D, dtype=torch.float32, device=dev)
    lse = torch.empty(B, len(heads), r1 - r0, dtype=torch.float32, device=dev)
    blk = max(1, min(r1 - r0, max_elems // max(1, Skv)))
    j = torch.arange(Skv, device=dev, dtype=torch.float32)
    for b in range(B):
        for hi, h in enumerate(heads):
            kf = k[b, :, h // group].float()  # [Skv, D]
            vf = v[b, :, h // group].float()
            for a in range(r0, r1, blk):
                e = min(r1, a + blk)
                qf = q[b, a:e, h].float()  # [n, D]
                s = (qf @ kf.t()) * sm_scale
                if alibi is not None:
                    s = s + float(alibi[h]) * j.view(1, Skv)
                if causal:
                    i = torch.arange(a, e, device=dev).view(-1, 1)
                    s = s.masked_fill(j.view(1, Skv) > (i + (Skv - Sq)), float("-inf"))
                m = s.amax(dim=-1, keepdim=True)
                m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
                p = torch.exp(s - m)
                l = p.sum(dim=-1, keepdim=True)
                l_safe = torch.where(l > 0, l, torch.ones_like(l))
                out[b, a - r0:e - r0, hi] = (p @ vf) / l_safe * (l > 0)
                lse[b, hi, a - r0:e - r0] = torch.where(l > 0, m + torch.log(l_safe),
                                                         torch.full_like(l, float("-inf"))).squeeze(-1)
    return out, lse
