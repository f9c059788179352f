"""Seeded input recipes for the golden attention fixtures.

Shared by ``make_golden.py`` (which runs the reference's own fp32 oracle,
``ref_attention`` in csrc/test_attention.py:41-93, on these inputs) and by the
tests that check the CPU oracle and the CUDA library against the stored
outputs.  Every input is generated on the CPU so that the fixtures are
reproducible without a GPU.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, asdict
from typing import List, Optional

import torch

DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


@dataclass
class GoldenCase:
    name: str
    kind: str  # "single" (one sequence, [S, H, D]) or "padded" ([B, S, H, D] + lens)
    dtype: str
    n_heads: int
    n_kv_heads: int
    head_dim: int
    q_len: int
    kv_len: int
    batch: int = 1
    q_lens: Optional[List[int]] = None
    kv_lens: Optional[List[int]] = None
    causal: bool = True
    sliding_window: int = -1
    logits_soft_cap: float = 0.0
    alibi: bool = False
    seed: int = 42
    recipe: str = "manual_seed"  # "manual_seed" (test_attention.py:109-112) or "generator"
    scale: float = 1.0  # multiplies q, k, v before the cast

    @property
    def sm_scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    def to_json(self):
        return asdict(self)


def alibi_slopes(n_heads: int) -> torch.Tensor:
    h = torch.arange(n_heads, dtype=torch.float64)
    return torch.pow(2.0, -8.0 * (h + 1.0) / n_heads).to(torch.float32)


def make_inputs(c: GoldenCase):
    """Returns q, k, v (CPU, in the case's dtype) and the ALiBi slopes or None.

    "manual_seed" reproduces the reference harness: torch.manual_seed(seed)
    then randn(q), randn(k), randn(v) directly in the dtype
    (csrc/test_attention.py:109-112), on the CPU generator.
    "generator" is the workload recipe: a torch.Generator seeded with `seed`,
    q, k, v drawn in fp32 in that order, scaled, then cast.
    """
    dt = DTYPES[c.dtype]
    if c.kind == "single":
        qs = (c.q_len, c.n_heads, c.head_dim)
        ks = (c.kv_len, c.n_kv_heads, c.head_dim)
    else:
        qs = (c.batch, c.q_len, c.n_heads, c.head_dim)
        ks = (c.batch, c.kv_len, c.n_kv_heads, c.head_dim)
    if c.recipe == "manual_seed":
        torch.manual_seed(c.seed)
        q = torch.randn(*qs, dtype=dt)
        k = torch.randn(*ks, dtype=dt)
        v = torch.randn(*ks, dtype=dt)
    else:
        g = torch.Generator().manual_seed(c.seed)
        q = torch.randn(*qs, generator=g, dtype=torch.float32)
        k = torch.randn(*ks, generator=g, dtype=torch.float32)
        v = torch.randn(*ks, generator=g, dtype=torch.float32)
        if c.scale != 1.0:
            q, k, v = q * c.scale, k * c.scale, v * c.scale
        q, k, v = q.to(dt), k.to(dt), v.to(dt)
    slopes = alibi_slopes(c.n_heads) if c.alibi else None
    return q, k, v, slopes


def _ref_suite() -> List[GoldenCase]:
    """The reference's 16-case parity suite (csrc/test_attention.py:143-201)."""
    out = []
    for dt in ("fp16", "bf16"):
        for hd in (64, 128):
            out.append(GoldenCase(f"mha_{dt}_h4_q256_hd{hd}", "single", dt, 4, 4, hd, 256, 256))
    for dt in ("fp16", "bf16"):
        out.append(GoldenCase(f"gqa_{dt}_h4_kv2", "single", dt, 4, 2, 128, 256, 256))
        out.append(GoldenCase(f"gqa_{dt}_h8_kv2", "single", dt, 8, 2, 128, 256, 256))
    for dt in ("fp16", "bf16"):
        out.append(GoldenCase(f"decode_{dt}_q1_kv256", "single", dt, 4, 2, 128, 1, 256))
        out.append(GoldenCase(f"decode_{dt}_q64_kv256", "single", dt, 4, 2, 128, 64, 256))
    for w in (32, 64, 128):
        out.append(GoldenCase(f"window_{w}", "single", "fp16", 4, 2, 128, 256, 256, sliding_window=w))
    for cap in (10.0, 50.0):
        out.append(GoldenCase(f"softcap_{int(cap)}", "single", "fp16", 4, 2, 128, 256, 256, logits_soft_cap=cap))
    return out


def _extended() -> List[GoldenCase]:
    """Paths the reference's oracle computes but its parity suite never runs."""
    return [
        # ALiBi through the single-sequence oracle (test_attention.py:73-77)
        GoldenCase("alibi_fp16_h4_q256_hd128", "single", "fp16", 4, 4, 128, 256, 256, alibi=True),
        GoldenCase("alibi_bf16_gqa_h8_kv2", "single", "bf16", 8, 2, 128, 200, 200, alibi=True),
        GoldenCase("alibi_window_softcap_fp16", "single", "fp16", 4, 2, 128, 160, 224,
                   alibi=True, sliding_window=48, logits_soft_cap=30.0),
        GoldenCase("ragged_bf16_q77_kv131_hd64", "single", "bf16", 2, 1, 64, 77, 131),
        # the CPU-runnable workload: B1 H8 S128 D64 fp32, causal, ALiBi, seed 0
        GoldenCase("c1_fp32_b1_h8_s128_d64_alibi", "padded", "fp32", 8, 8, 64, 128, 128,
                   alibi=True, seed=0, recipe="generator"),
        # padded, non-causal prefill (padded-prefill workload, small): keys past len masked
        GoldenCase("padded_noncausal_fp16_alibi", "padded", "fp16", 4, 4, 64, 96, 96, batch=2,
                   q_lens=[70, 96], kv_lens=[70, 96], causal=False, alibi=True, seed=1,
                   recipe="generator"),
        # batched decode (decode workload, small): q_len 1, padded cache, GQA
        GoldenCase("decode_padded_bf16_alibi_gqa", "padded", "bf16", 8, 2, 128, 1, 300, batch=3,
                   q_lens=[1, 1, 1], kv_lens=[1, 150, 300], causal=True, alibi=True, seed=2,
                   recipe="generator"),
        GoldenCase("decode_padded_bf16_alibi_mha", "padded", "bf16", 8, 8, 128, 1, 520, batch=2,
                   q_lens=[1, 1], kv_lens=[519, 257], causal=True, alibi=True, seed=3,
                   recipe="generator"),
    ]


def all_cases() -> List[GoldenCase]:
    return _ref_suite() + _extended()


def case_by_name(name: str) -> GoldenCase:
    for c in all_cases():
        if c.name == name:
            return c
    raise KeyError(name)
