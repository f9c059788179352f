"""Log-sum-exp merge of attention partials, restated in torch (fp32).

TEST INFRASTRUCTURE ONLY (the checker for the KV-split merge kernel and the
CPU stand-in for it in the multi-rank host-logic tests); the product path
merges with the library's kernel.

A query row's attention over keys K = K_1 u ... u K_n follows from the
partials (O_c, lse_c) over each K_c: m = max_c lse_c, w_c = exp(lse_c - m),
O = sum_c w_c O_c / sum_c w_c, lse = m + log(sum_c w_c) -- the running max /
running sum rescale of the reference's online softmax (softmax.h:53-110)
applied across key shards.  A partial with lse = -inf contributes nothing.
"""

from __future__ import annotations

from typing import Sequence

import torch


def merge_partials(outs: Sequence[torch.Tensor], lses: Sequence[torch.Tensor]):
    """outs: [B, S, H, D] each; lses: [B, H, S] fp32 natural log (-inf where a
    row saw no key).  Returns (O fp32 [B, S, H, D], lse [B, H, S])."""
    lse = torch.stack([l.float() for l in lses], 0)  # [n, B, H, S]
    m = lse.amax(0)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.where(torch.isfinite(lse), torch.exp(lse - m_safe), torch.zeros_like(lse))
    wsum = w.sum(0)
    num = None
    for o, wi in zip(outs, w):
        term = torch.where(wi.permute(0, 2, 1).unsqueeze(-1) > 0, o.float() * wi.permute(0, 2, 1).unsqueeze(-1),
                           torch.zeros((), dtype=torch.float32, device=o.device))
        num = term if num is None else num + term
    inv = torch.where(wsum > 0, 1.0 / wsum, torch.zeros_like(wsum))
    out = num * inv.permute(0, 2, 1).unsqueeze(-1)
    lse_out = torch.where(wsum > 0, m_safe + torch.log(wsum), torch.full_like(m, float("-inf")))
    return out, lse_out


def merge_row_parts(parts, B: int, S: int, H: int, D: int, device="cpu"):
    """Partials that each cover output rows [row_lo, row_hi): parts are
    (o [B, n, H, D], lse [B, H, n], row_lo, row_hi), n = row_hi - row_lo.
    Rows outside a part's range get no term from it.  Returns (O fp32
    [B, S, H, D], lse [B, H, S])."""
    outs, lses = [], []
    for o, l, lo, hi in parts:
        fo = torch.zeros(B, S, H, D, dtype=torch.float32, device=device)
        fl = torch.full((B, H, S), float("-inf"), dtype=torch.float32, device=device)
        if hi > lo:
            fo[:, lo:hi] = o.float().to(device)
            fl[:, :, lo:hi] = l.float().to(device)
        outs.append(fo)
        lses.append(fl)
    if not outs:
        return (torch.zeros(B, S, H, D, dtype=torch.float32, device=device),
                torch.full((B, H, S), float("-inf"), dtype=torch.float32, device=device))
    return merge_partials(outs, lses)
