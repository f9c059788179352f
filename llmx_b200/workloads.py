"""The attention workloads this engine is measured on (five configurations
of the reference's use cases plus a head_dim 256 prefill), with their
seeded synthetic inputs and algorithmic work counts.

Recipe (shared by the tests and the benchmark): a CPU ``torch.Generator``
seeded with the workload's seed draws the per-sequence lengths first; q, k, v
are then drawn from N(0, 1) in fp32 in that order (on the CPU for the small
workloads, with a generator on the target device for the large ones), scaled
and cast.  ALiBi slopes are m_h = 2^(-8(h+1)/H); sm_scale = 1/sqrt(D).

Work counts never include masked, padded or causally skipped work:
FLOPs = 4 * D * (number of visible (query, key) pairs) per head, and decode
bytes = the K/V rows actually read plus q, o, lengths and slopes.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    description: str
    dtype: torch.dtype
    batch: int
    n_heads: int
    n_kv_heads: int
    q_len: int  # padded extent of the query axis
    kv_len: int  # padded extent of the key axis
    head_dim: int
    causal: bool
    alibi: bool
    scale: float = 1.0
    lens: Optional[tuple] = None  # (low, high_exclusive) of randint, or None = full
    lens_apply_to_q: bool = False  # padded prefill: q_lens = kv_lens
    seed: int = 0
    device_inputs: bool = False  # draw q/k/v on the device (large workloads)

    @property
    def sm_scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    @property
    def is_decode(self) -> bool:
        return self.q_len == 1


WORKLOADS = {
    "cpu_fp32_b1_h8_s128_d64": Workload(
        "cpu_fp32_b1_h8_s128_d64", "CPU-runnable MHA: B1 H8 S128 D64 fp32, causal, ALiBi",
        torch.float32, 1, 8, 8, 128, 128, 64, causal=True, alibi=True),
    "padded_prefill_fp16_b4_h16_s1024_d64": Workload(
        "padded_prefill_fp16_b4_h16_s1024_d64",
        "Padded prefill: B4 H16 S<=1024 D64 fp16, lens U[512,1024], non-causal, ALiBi",
        torch.float16, 4, 16, 16, 1024, 1024, 64, causal=False, alibi=True, lens=(512, 1025),
        lens_apply_to_q=True),
    "llama7b_prefill_bf16_b8_h32_s2048_d128": Workload(
        "llama7b_prefill_bf16_b8_h32_s2048_d128",
        "Llama-7B-shaped causal prefill: B8 H32 S2048 D128 bf16, QKV*0.5",
        torch.bfloat16, 8, 32, 32, 2048, 2048, 128, causal=True, alibi=False, scale=0.5,
        device_inputs=True),
    "bloom_decode_bf16_b64_h32_kv4096_d128": Workload(
        "bloom_decode_bf16_b64_h32_kv4096_d128",
        "BLOOM-style batched decode: B64 H32 Sq1 KV<=4096 D128 bf16, ALiBi, padded cache",
        torch.bfloat16, 64, 32, 32, 1, 4096, 128, causal=True, alibi=True, lens=(256, 4097),
        device_inputs=True),
    "gemma_prefill_bf16_b2_h16_s4096_d256": Workload(
        "gemma_prefill_bf16_b2_h16_s4096_d256",
        "Head-dim-256 causal prefill (Gemma-7B-shaped heads): B2 H16 S4096 D256 bf16",
        torch.bfloat16, 2, 16, 16, 4096, 4096, 256, causal=True, alibi=False, device_inputs=True),
    "long_prefill_bf16_b1_h32_s32768_d128": Workload(
        "long_prefill_bf16_b1_h32_s32768_d128",
        "Long-context causal prefill: B1 H32 S32768 D128 bf16, ALiBi",
        torch.bfloat16, 1, 32, 32, 32768, 32768, 128, causal=True, alibi=True, device_inputs=True),
}


def alibi_slopes(n_heads: int, device="cpu") -> torch.Tensor:
    h = torch.arange(n_heads, dtype=torch.float64)
    return torch.pow(2.0, -8.0 * (h + 1.0) / n_heads).to(torch.float32).to(device)


def draw_lengths(w: Workload, seed: Optional[int] = None) -> List[int]:
    g = torch.Generator().manual_seed(w.seed if seed is None else seed)
    if w.lens is None:
        return [w.kv_len] * w.batch
    return torch.randint(w.lens[0], w.lens[1], (w.batch,), generator=g).tolist()


@dataclass
class Inputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    kv_lens_list: List[int]
    q_lens_list: List[int]
    q_lens: Optional[torch.Tensor] = None
    kv_lens: Optional[torch.Tensor] = None
    alibi: Optional[torch.Tensor] = None
    extra: dict = field(default_factory=dict)


def make_inputs(w: Workload, device="cuda", seed: Optional[int] = None, batch: Optional[int] = None) -> Inputs:
    """Seeded inputs of workload `w` on `device` ([B, S, H, D] layout).

    `batch` overrides the batch size (used to give each rank its own shard of
    a larger job); `seed` overrides the workload seed.
    """
    if batch is not None and batch != w.batch:
        from dataclasses import replace

        w = replace(w, batch=batch)
    seed = w.seed if seed is None else seed
    g = torch.Generator().manual_seed(seed)
    if w.lens is None:
        kv_lens = [w.kv_len] * w.batch
    else:
        kv_lens = torch.randint(w.lens[0], w.lens[1], (w.batch,), generator=g).tolist()
    q_lens = list(kv_lens) if w.lens_apply_to_q else [w.q_len] * w.batch
    qs = (w.batch, w.q_len, w.n_heads, w.head_dim)
    ks = (w.batch, w.kv_len, w.n_kv_heads, w.head_dim)
    if w.device_inputs and torch.device(device).type == "cuda":
        gd = torch.Generator(device=device).manual_seed(seed)
        draw = lambda shape: torch.randn(shape, generator=gd, device=device, dtype=torch.float32)  # noqa: E731
    else:
        draw = lambda shape: torch.randn(shape, generator=g, dtype=torch.float32)  # noqa: E731
    out = []
    for shape in (qs, ks, ks):
        t = draw(shape)
        if w.scale != 1.0:
            t.mul_(w.scale)
        out.append(t.to(w.dtype).to(device))
        del t
    q, k, v = out
    inp = Inputs(q, k, v, kv_lens, q_lens)
    if w.lens is not None:
        inp.kv_lens = torch.tensor(kv_lens, dtype=torch.int32, device=device)
        if w.lens_apply_to_q:
            inp.q_lens = torch.tensor(q_lens, dtype=torch.int32, device=device)
    if w.alibi:
        inp.alibi = alibi_slopes(w.n_heads, device)
    return inp


def visible_pairs(q_len: int, kv_len: int, causal: bool, window: int = -1) -> int:
    """Number of (query, key) pairs the mask leaves visible in one sequence."""
    if q_len <= 0 or kv_len <= 0:
        return 0
    total = 0
    off = kv_len - q_len
    if not causal and window < 0:
        return q_len * kv_len
    for i in range(q_len):
        hi = min(kv_len - 1, i + off) if causal else kv_len - 1
        lo = max(0, i + off - window) if window >= 0 else 0
        if hi >= lo:
            total += hi - lo + 1
    return total


def flops(w: Workload, q_lens: List[int], kv_lens: List[int]) -> int:
    pairs = sum(visible_pairs(ql, kl, w.causal) for ql, kl in zip(q_lens, kv_lens))
    return 4 * w.head_dim * w.n_heads * pairs


def decode_bytes(w: Workload, kv_lens: List[int]) -> int:
    """Algorithmic HBM bytes of one decode step: every visible K/V row once,
    plus q, o, the length array and the slopes."""
    es = torch.tensor([], dtype=w.dtype).element_size()
    kv = sum(kv_lens) * w.n_kv_heads * w.head_dim * 2 * es
    qo = 2 * w.batch * w.n_heads * w.head_dim * es
    meta = 4 * w.batch + (4 * w.n_heads if w.alibi else 0)
    return kv + qo + meta
