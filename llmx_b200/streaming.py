"""Attention over host-resident (pinned) tensors, with the copies overlapped.

``attention_from_host`` is the call a user makes when q, k, v live in host
memory and the output is wanted back there: the batch is cut into chunks and
each chunk's host->device copy, kernel and device->host copy run on three
streams, so that chunk i+1 uploads while chunk i computes and chunk i-1
downloads (PCIe is full duplex, so the two copy directions overlap too).
The reference has no host-memory entry point: its binding takes device
tensors only (csrc/llmx_bind.cpp:23-25); its copies are synchronous
cudaMemcpy calls behind llmx_copy (src/tensor.cpp:84-106).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops


def plan_pieces(ranges, seq_len: int, tail_pieces: int):
    """The pipeline's work pieces (b0, b1, r0, r1): batch elements [b0, b1),
    query rows [r0, r1).  Every chunk of `ranges` is one piece over all rows,
    except that with tail_pieces > 1 (causal self-attention only) the last
    batch element is cut into up to `tail_pieces` row ranges with boundaries
    on multiples of 128 rows (the kernel's query tile), so that a row's result
    does not depend on the cut; sequences shorter than 2 * tail_pieces * 128
    rows are not cut.  The pieces cover every (batch, row) once, in order."""
    tail = tail_pieces if tail_pieces > 1 and seq_len >= 2 * tail_pieces * 128 else 1
    pieces = []
    for i, (a, b) in enumerate(ranges):
        if tail > 1 and i == len(ranges) - 1:
            if b - a > 1:
                pieces.append((a, b - 1, 0, seq_len))
                a = b - 1
            rows = [round(p * seq_len / tail / 128) * 128 for p in range(tail)] + [seq_len]
            pieces += [(a, b, r0, r1) for r0, r1 in zip(rows, rows[1:]) if r1 > r0]
        else:
            pieces.append((a, b, 0, seq_len))
    return pieces


class HostAttention:
    """Device buffers, streams and events for repeated host-to-host attention
    calls of one shape (allocated once, reused by every call).

    The batch is cut into `chunks` pieces.  What is left after the last
    upload -- that piece's kernel and download -- is the pipeline's tail, so
    for causal self-attention (q_len == kv_len, no per-sequence lengths) the
    last batch element is further cut into `tail_pieces` row ranges: rows
    [r0, r1) see only keys [0, r1), so each piece uploads its own q / k / v
    rows, computes, and downloads its output rows while the next uploads.
    A row's result does not depend on the cut (the same key blocks in the
    same order)."""

    def __init__(self, q_host: torch.Tensor, k_host: torch.Tensor, device, chunks: int = 4, tail_pieces: int = 2):
        if q_host.dim() != 4 or k_host.dim() != 4:
            raise RuntimeError("attention_from_host takes 4-D [batch, seq, heads, head_dim] tensors")
        B = q_host.shape[0]
        self.device = torch.device(device)
        self.chunks = max(1, min(chunks, B))
        bounds = [round(i * B / self.chunks) for i in range(self.chunks + 1)]
        self.ranges = [(a, b) for a, b in zip(bounds, bounds[1:]) if b > a]
        S = q_host.shape[1]
        self.tail_pieces = max(1, int(tail_pieces)) if S == k_host.shape[1] else 1
        self.qd = torch.empty(q_host.shape, dtype=q_host.dtype, device=self.device)
        self.kd = torch.empty(k_host.shape, dtype=k_host.dtype, device=self.device)
        self.vd = torch.empty(k_host.shape, dtype=k_host.dtype, device=self.device)
        self.od = torch.empty_like(self.qd)
        self.up = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.down = torch.cuda.Stream(self.device)

    def __call__(self, out_host, q_host, k_host, v_host, sm_scale: float, stream: Optional[torch.cuda.Stream] = None,
                 **kw) -> None:
        """Enqueues the whole pipeline after the work already on `stream`
        (default: the current stream) and makes `stream` wait for its end;
        out_host is complete once `stream` is synchronised."""
        if not (q_host.is_pinned() and k_host.is_pinned() and v_host.is_pinned() and out_host.is_pinned()):
            raise RuntimeError("attention_from_host needs pinned host tensors (tensor.pin_memory())")
        caller = stream or torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(caller)
        for s in (self.up, self.comp, self.down):
            s.wait_event(start)
        S = q_host.shape[1]
        row_cut = (kw.get("causal", True) and kw.get("q_lens") is None and kw.get("kv_lens") is None)
        pieces = plan_pieces(self.ranges, S, self.tail_pieces if row_cut else 1)
        for a, b, r0, r1 in pieces:
            with torch.cuda.stream(self.up):
                self.qd[a:b, r0:r1].copy_(q_host[a:b, r0:r1], non_blocking=True)
                self.kd[a:b, r0:r1].copy_(k_host[a:b, r0:r1], non_blocking=True)
                self.vd[a:b, r0:r1].copy_(v_host[a:b, r0:r1], non_blocking=True)
                up_done = torch.cuda.Event()
                up_done.record(self.up)
            self.comp.wait_event(up_done)
            with torch.cuda.stream(self.comp):
                kwc = dict(kw)
                for name in ("q_lens", "kv_lens"):
                    if kwc.get(name) is not None:
                        kwc[name] = kwc[name][a:b]  # per-sequence lengths of the chunk
                # a row piece [r0, r1) of causal self-attention sees keys [0, r1)
                ops.single_mha_attention_half(self.od[a:b, r0:r1], self.qd[a:b, r0:r1], self.kd[a:b, :r1],
                                              self.vd[a:b, :r1], sm_scale, **kwc)
                comp_done = torch.cuda.Event()
                comp_done.record(self.comp)
            self.down.wait_event(comp_done)
            with torch.cuda.stream(self.down):
                out_host[a:b, r0:r1].copy_(self.od[a:b, r0:r1], non_blocking=True)
        end = torch.cuda.Event()
        end.record(self.down)
        caller.wait_event(end)
        # the device buffers are reused by the next call on these streams
        for s in (self.up, self.comp):
            s.wait_event(end)


def attention_from_host(out_host, q_host, k_host, v_host, sm_scale: float, *, device="cuda", chunks: int = 4,
                        tail_pieces: int = 2, **kw) -> None:
    """One host-to-host attention call (allocates its device buffers; use
    HostAttention to reuse them across calls).  Blocks until out_host is
    written.  Keyword arguments are those of single_mha_attention_half
    (alibi_slopes, causal, q_lens, kv_lens as device tensors)."""
    h = HostAttention(q_host, k_host, device, chunks, tail_pieces)
    h(out_host, q_host, k_host, v_host, sm_scale, **kw)
    torch.cuda.current_stream(h.device).synchronize()
