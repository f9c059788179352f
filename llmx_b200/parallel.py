"""Multi-GPU partitioning of the attention forward (one process per GPU).

Three ways the work splits across the GPUs of one node:

* **batch x head shards** (independent units, no communication): every
  (batch, head) pair is an independent attention problem.  ``shard_units``
  gives each rank a contiguous slice of the flattened units of equal count,
  ``shard_units_weighted`` one of equal work (sequences of unequal length),
  and ``run_units`` runs the kernel on such a slice (one launch per batch run).
* **head split** of one long sequence (``head_range``): each rank takes a
  contiguous block of heads, whole GQA groups, and runs the kernel on it; no
  communication.
* **KV split** of one long sequence (``KVSplitPlan`` + ``kv_split_attention``):
  rank r holds a share of the keys.  Under the causal mask a query row below
  the rank's first key sees none of them, so the rank computes its partial
  (O_r, lse_r) only for the rows from ``plan.first_row(r)`` on.  The output
  rows are dealt in equal slices, one per rank; each rank sends every other
  rank the rows of its partial that fall in that rank's slice (NCCL
  point-to-point in one group), and merges the partials of its own slice
  exactly with the log-sum-exp rule

      m = max_r lse_r,  O = sum_r exp(lse_r - m) O_r / sum_r exp(lse_r - m)

  in one kernel.  The result is row-sharded (``output="sharded"``) or, after
  an all-gather of the slices, on every rank (``output="replicated"``).

Every collective or point-to-point step is derived from the plan, which
every rank computes identically, so all ranks issue matching NCCL calls
whatever their local key count (a rank without keys sends nothing and still
receives its slice).

The reference has no multi-GPU code; its kernel already streams keys through
an online softmax inside one SM (single_mha_kernel.cuh:294-340), and the
merge here is the same running-max / running-sum algebra applied across
shards instead of across blocks (softmax.h:53-110).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib, ops

# ---------------------------------------------------------------- unit shards


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


def shard_units_weighted(weights: Sequence[float], heads: int, world: int, rank: int,
                         align: int = 1) -> Tuple[int, int]:
    """Contiguous range [start, end) of flattened (batch, head) units for
    `rank`, balanced on work instead of unit count: every head of batch
    element b weighs weights[b] (its key length for decode, its visible
    (query, key) pairs for prefill).  Boundaries fall on multiples of
    `align` units (whole GQA groups); each rank's range ends at the first
    boundary where the running weight reaches (rank + 1) / world of the
    total, so ranges cover every unit exactly once (some may be empty when
    there are fewer granules than ranks)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if align < 1 or heads % align:
        raise ValueError("align must divide heads")
    units = len(weights) * heads
    n_gran = units // align
    gw = [float(weights[(i * align) // heads]) * align for i in range(n_gran)]
    total = sum(gw)
    if total <= 0:
        g0, g1 = shard_units(1, n_gran, world, rank)
        return g0 * align, g1 * align

    def edge(r: int) -> int:
        if r <= 0:
            return 0
        if r >= world:
            return n_gran
        target, acc = total * r / world, 0.0
        for i, x in enumerate(gw):
            if acc + x / 2 >= target:  # the granule goes to the rank holding most of it
                return i
            acc += x
        return n_gran

    return edge(rank) * align, edge(rank + 1) * align


def launch_granule(batch: int, heads: int, world: int, group: int = 1) -> int:
    """The coarsest unit granule for ``shard_units_weighted`` that still
    gives every rank something to do: whole sequences (`heads` units) when
    there are at least as many sequences as ranks, else the largest block of
    whole GQA groups dividing `heads` with batch * heads / granule >= world.
    Ranges of whole granules cut a rank's units into fewer launches (one per
    run of whole sequences or one head block), which is what a small job's
    time depends on: each launch has a fixed cost and fills the GPU only
    partly."""
    if world < 1 or heads % group:
        raise ValueError("world >= 1 and group dividing heads required")
    g = heads
    while g > group and (batch * heads) // g < world:
        g //= 2
        while g > group and (heads % g or g % group):
            g -= 1
    return max(group, g)


def unit_runs(start: int, end: int, heads: int) -> List[Tuple[int, int, int, int]]:
    """The unit range [start, end) as launches: (b0, b1, h0, h1) boxes of whole
    head runs, at most three (a partial first batch, whole batches, a partial
    last batch)."""
    runs = []
    u = start
    while u < end:
        b, h = divmod(u, heads)
        if h == 0 and end - u >= heads:
            nb = (end - u) // heads
            runs.append((b, b + nb, 0, heads))
            u += nb * heads
        else:
            h1 = min(heads, h + (end - u))
            runs.append((b, b + 1, h, h1))
            u += h1 - h
    return runs


def run_units(out, q, k, v, start: int, end: int, sm_scale: float, *, alibi_slopes=None, **kw) -> int:
    """Attention of the (batch, head) units [start, end) of [B, S, H, D] tensors,
    written into the same units of `out`; other units are untouched.  Returns
    the number of launches.  With GQA every head run must cover whole groups."""
    H, Hkv = q.shape[2], k.shape[2]
    g = H // Hkv
    n = 0
    for b0, b1, h0, h1 in unit_runs(start, end, H):
        if h0 % g or h1 % g:
            raise ValueError("a unit shard must hold whole GQA groups")
        a = None if alibi_slopes is None else alibi_slopes[h0:h1]
        kwr = dict(kw)
        for name in ("q_lens", "kv_lens"):
            if kwr.get(name) is not None:
                kwr[name] = kwr[name][b0:b1]  # per-sequence lengths of the run's batch elements
        ops.single_mha_attention_half(out[b0:b1, :, h0:h1], q[b0:b1, :, h0:h1], k[b0:b1, :, h0 // g:h1 // g],
                                      v[b0:b1, :, h0 // g:h1 // g], sm_scale, alibi_slopes=a, **kwr)
        n += 1
    return n


def head_range(n_heads: int, world: int, rank: int, group: int = 1) -> Tuple[int, int]:
    """Contiguous heads [h0, h1) of `rank` when whole GQA groups of `group`
    heads are dealt over `world` ranks (sizes differ by at most one group)."""
    if n_heads % group:
        raise ValueError("group must divide n_heads")
    g0, g1 = shard_units(1, n_heads // group, world, rank)
    return g0 * group, g1 * group


# ---------------------------------------------------------------- key shards


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

    Range boundaries are multiples of `align`, and when seq_len >= world *
    align every rank gets at least one align block (the balanced boundaries
    are clamped into [r * align, seq_len - (world - r) * align]).  Shorter
    sequences are too short to split that finely: the ranges then come from
    the same rule over the ranks that get a block each, the last ones empty.
    The ranges cover every key exactly once.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    blocks = -(-seq_len // align)
    eff = max(1, min(world, blocks))  # ranks that can get at least one block
    if rank >= eff:
        return seq_len, seq_len
    total = seq_len * (seq_len + 1) / 2
    b = 2 * seq_len + 1

    def bound(r: int) -> int:
        if r <= 0:
            return 0
        if r >= eff:
            return seq_len
        # smallest x with x * seq_len - x * (x - 1) / 2 >= r * total / eff
        x = (b - math.sqrt(max(0.0, b * b - 8 * r * total / eff))) / 2
        x = int(round(x / align)) * align
        return max(r * align, min(x, seq_len - (eff - r) * align, seq_len))

    return bound(rank), bound(rank + 1)


# Work-item geometry of the tensor-core prefill kernel: items of 256 query
# rows (two 128-row tiles) over key blocks of 128, and the cost of one item's
# start and epilogue in key-block units.  With 1.5 the per-rank kernel times
# of an 8-way split of a 32768-token causal sequence, measured on B200, came
# out within 6% of each other (the pair-balanced split: within 11%).
ITEM_ROWS = 256
KEY_BLOCK = 128
ITEM_COST = 1.5


def key_range_cost(a: int, b: int, q_len: int, kv_len: int, *, item_rows: int = ITEM_ROWS,
                   block: int = KEY_BLOCK, item_cost: float = ITEM_COST) -> float:
    """Modelled kernel time, in key-block units per head, of the causal
    partial of keys [a, b) (bottom-right aligned): its rows are those from
    the first that sees key a; each item of `item_rows` rows costs
    `item_cost` plus one unit per key block its last row sees."""
    if b <= a:
        return 0.0
    shift = kv_len - q_len
    r0 = max(0, min(q_len, a - shift))
    n_items = -(-(q_len - r0) // item_rows)
    total = 0.0
    for i in range(n_items):
        last = min(q_len - 1, r0 + (i + 1) * item_rows - 1)
        seen = min(b, last + shift + 1) - a
        if seen > 0:
            total += item_cost + -(-seen // block)
    return total


def balanced_key_ranges(seq_len: int, world: int, *, align: int = KEY_BLOCK,
                        item_cost: float = ITEM_COST) -> List[Tuple[int, int]]:
    """One contiguous key range per rank for a causal self-attention split,
    chosen to minimise the largest ``key_range_cost`` over the ranks (the
    kernel-time balance: a rank holding late keys computes a causal
    triangle of short items, one holding early keys long rectangles).

    Boundaries are multiples of `align` (the last range ends at seq_len);
    every rank gets at least one block when seq_len >= world * align, else
    the trailing ranks get empty ranges.  The ranges cover every key once.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    n_blk = -(-seq_len // align)
    eff = max(1, min(world, n_blk))
    pos = [min(seq_len, i * align) for i in range(n_blk + 1)]
    cost = lambda i, j: key_range_cost(pos[i], pos[j], seq_len, seq_len, item_cost=item_cost)

    def cut(limit: float) -> Optional[List[int]]:
        # greedy: each range takes as many blocks as fit under `limit`,
        # leaving at least one block for every later rank
        edges = [0]
        for r in range(eff - 1):
            i = edges[-1]
            lo, hi = i + 1, n_blk - (eff - 1 - r)
            if lo > hi or cost(i, lo) > limit:
                return None
            while lo < hi:  # largest j in [lo, hi] with cost(i, j) <= limit
                mid = (lo + hi + 1) // 2
                if cost(i, mid) <= limit:
                    lo = mid
                else:
                    hi = mid - 1
            edges.append(lo)
        if cost(edges[-1], n_blk) > limit:
            return None
        return edges + [n_blk]

    lo_t, hi_t = 0.0, cost(0, n_blk)
    best = cut(hi_t) if eff == 1 else None
    for _ in range(60):
        if eff == 1:
            break
        mid = (lo_t + hi_t) / 2
        e = cut(mid)
        if e is None:
            lo_t = mid
        else:
            hi_t, best = mid, e
        if hi_t - lo_t < 1e-3:
            break
    if best is None:
        best = cut(hi_t)
    ranges = [(pos[best[r]], pos[best[r + 1]]) for r in range(eff)]
    return ranges + [(seq_len, seq_len)] * (world - eff)


def kv_split_ranges(seq_len: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """The key ranges of `rank` for a causal KV split over `world` ranks: one
    contiguous, work-balanced range (``causal_key_range``), or none for a
    rank left without keys by a sequence shorter than world * 16 keys."""
    a, b = causal_key_range(seq_len, world, rank)
    return [(a, b)] if b > a else []


@dataclass(frozen=True)
class KVSplitPlan:
    """Who holds which keys and who owns which output rows, for one sequence
    of `q_len` queries over `kv_len` keys split over `world` ranks.

    chunks[r]: the key ranges [a, b) rank r holds (ascending).  Output rows
    are dealt in slices of `slice_rows` (the last one shorter or empty).
    Under the causal mask (bottom-right: row i sees key j <= i + kv_len -
    q_len) a rank computes its partial only for rows >= first_row(r)."""

    q_len: int
    kv_len: int
    world: int
    chunks: Tuple[Tuple[Tuple[int, int], ...], ...]
    causal: bool = True

    @classmethod
    def contiguous(cls, seq_len: int, world: int, causal: bool = True, balance: str = "kernel") -> "KVSplitPlan":
        """One key range per rank: balanced on the kernel's modelled time
        (``balanced_key_ranges``, the default) or on visible causal pairs
        (``balance="pairs"``, ``kv_split_ranges``); even ranges without the
        causal mask."""
        if not causal:
            ch = tuple(tuple(_even_range(seq_len, world, r)) for r in range(world))
        elif balance == "kernel":
            ch = tuple(((a, b),) if b > a else () for a, b in balanced_key_ranges(seq_len, world))
        elif balance == "pairs":
            ch = tuple(tuple(kv_split_ranges(seq_len, world, r)) for r in range(world))
        else:
            raise ValueError("balance must be 'kernel' or 'pairs'")
        return cls(seq_len, seq_len, world, ch, causal)

    @classmethod
    def zigzag(cls, seq_len: int, world: int, causal: bool = True, align: int = 128) -> "KVSplitPlan":
        """Two chunks per rank (``zigzag_chunks``)."""
        ch = tuple(tuple(zigzag_chunks(seq_len, world, r, align)) for r in range(world))
        return cls(seq_len, seq_len, world, ch, causal)

    @property
    def slice_rows(self) -> int:
        s = -(-self.q_len // self.world)
        return -(-s // 16) * 16

    def row_slice(self, rank: int) -> Tuple[int, int]:
        lo = min(self.q_len, rank * self.slice_rows)
        return lo, min(self.q_len, lo + self.slice_rows)

    def chunk_first_row(self, key_start: int) -> int:
        """First query row that sees key `key_start` (q_len if none)."""
        if not self.causal:
            return 0
        return max(0, min(self.q_len, key_start - (self.kv_len - self.q_len)))

    def first_row(self, rank: int) -> int:
        rows = [self.chunk_first_row(a) for a, b in self.chunks[rank] if b > a]
        return min(rows) if rows else self.q_len


def _even_range(seq_len: int, world: int, rank: int) -> List[Tuple[int, int]]:
    a, b = shard_units(1, seq_len, world, rank)
    return [(a, b)] if b > a else []


# ---------------------------------------------------------------- KV split


class CudaOps:
    """The kernels of the KV split on this GPU: attention over one key chunk
    (libllmx_attn.so's forward with kv_offset / kv_total) and the log-sum-exp
    merge (llmx_attn_lse_merge)."""

    def attend(self, o, lse, q, k, v, sm_scale, *, alibi_slopes, causal, sliding_window, kv_offset, kv_total):
        ops.single_mha_attention_half(o, q, k, v, sm_scale, sliding_window, alibi_slopes=alibi_slopes,
                                      causal=causal, lse=lse, kv_offset=kv_offset, kv_total=kv_total)

    def merge(self, parts, out, lse_out):
        """parts: (o [B, n, H, D], lse [B, H, n], row_lo, row_hi) with n =
        row_hi - row_lo, rows counted in `out`'s row axis."""
        raw = []
        for o, l, lo, hi in parts:
            if o.dtype != out.dtype or l.dtype != torch.float32 or o.stride(-1) != 1 or l.stride(-1) != 1:
                raise RuntimeError("merge parts: O in the output dtype with unit head_dim stride, fp32 lse")
            raw.append((o.data_ptr(), (o.stride(0), o.stride(1), o.stride(2)), l.data_ptr(), (l.stride(0), l.stride(1)),
                        lo, hi))
        self.merge_raw(raw, out, lse_out)

    def merge_raw(self, parts, out, lse_out):
        """As merge, with each part given as (o address, o element strides
        (batch, row, head), lse address, lse strides (batch, head), row_lo,
        row_hi): device memory the caller guarantees is live."""
        B, S, H, D = out.shape
        if out.dtype not in (torch.float16, torch.bfloat16):
            raise RuntimeError("the KV-split merge takes fp16 or bf16 partials")
        arr = (_lib.MergePart * max(1, len(parts)))()
        for i, (optr, ost_p, lptr, lst_p, lo, hi) in enumerate(parts):
            arr[i].o, arr[i].lse = optr, lptr
            arr[i].o_stride[:] = tuple(int(x) for x in ost_p)
            arr[i].lse_stride[:] = tuple(int(x) for x in lst_p)
            arr[i].row_lo, arr[i].row_hi = int(lo), int(hi)
        ost = (ctypes.c_int64 * 3)(out.stride(0), out.stride(1), out.stride(2))
        dt = _lib.DTYPE["bf16" if out.dtype == torch.bfloat16 else "fp16"]
        stream = ctypes.c_void_p(torch.cuda.current_stream(out.device).cuda_stream)
        _lib.check(_lib.load().llmx_attn_lse_merge(len(parts), arr, dt, B, S, H, D, out.data_ptr(), ost,
                                                   None if lse_out is None else lse_out.data_ptr(), stream))


def _mark(timings, name, device):
    if timings is not None and device.type == "cuda":
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(device))
        timings.append((name, ev))


def local_partial(q, k_chunks, v_chunks, plan: KVSplitPlan, rank: int, sm_scale: float, *, alibi_slopes=None,
                  sliding_window: int = -1, backend=None):
    """This rank's partial over its keys: (O [B, q_len - row0, H, D],
    lse [B, H, q_len - row0], row0) for the rows row0 = plan.first_row(rank)
    on.  Each chunk is computed for the rows that can see it (one kernel
    launch per chunk) and several chunks are merged into one partial."""
    be = backend or CudaOps()
    B, Sq, H, D = q.shape
    dev = q.device
    mine = plan.chunks[rank]
    if len(k_chunks) != len(mine) or len(v_chunks) != len(mine):
        raise ValueError("one k / v chunk per key range of this rank")
    row0 = plan.first_row(rank)
    pieces = []
    for (a, b), kc, vc in zip(mine, k_chunks, v_chunks):
        if kc.shape[1] != b - a or vc.shape[1] != b - a:
            raise ValueError("chunk length differs from the plan's key range")
        r0 = plan.chunk_first_row(a)
        if b <= a or r0 >= Sq:
            continue
        o = torch.empty(B, Sq - r0, H, D, dtype=q.dtype, device=dev)
        l = torch.empty(B, H, Sq - r0, dtype=torch.float32, device=dev)
        be.attend(o, l, q[:, r0:], kc, vc, sm_scale, alibi_slopes=alibi_slopes, causal=plan.causal,
                  sliding_window=sliding_window, kv_offset=a, kv_total=plan.kv_len)
        pieces.append((o, l, r0 - row0, Sq - row0))
    if len(pieces) == 1:
        return pieces[0][0], pieces[0][1], row0
    part_o = torch.empty(B, Sq - row0, H, D, dtype=q.dtype, device=dev)
    part_l = torch.empty(B, H, Sq - row0, dtype=torch.float32, device=dev)
    if Sq > row0:
        be.merge(pieces, part_o, part_l)
    return part_o, part_l, row0


def slice_part(part_o, part_l, row0: int, plan: KVSplitPlan, src: int, dst: int):
    """The rows of rank `src`'s partial (from ``local_partial``) that fall in
    rank `dst`'s row slice, as (O view, lse view, row_lo, row_hi) with rows
    counted inside the slice, or None when there are none."""
    lo, hi = plan.row_slice(dst)
    a = max(lo, row0, plan.first_row(src))
    if hi <= a:
        return None
    return part_o[:, a - row0:hi - row0], part_l[:, :, a - row0:hi - row0], a - lo, hi - lo


def merge_slice(parts, plan: KVSplitPlan, rank: int, like: torch.Tensor, *, rows: Optional[int] = None,
                backend=None):
    """Merges the partials of rank `rank`'s row slice: returns (O [B, rows, H, D],
    lse [B, H, rows]) with rows = the slice length unless given (padding rows
    past the slice are left unwritten)."""
    be = backend or CudaOps()
    B, _, H, D = like.shape
    lo, hi = plan.row_slice(rank)
    rows = hi - lo if rows is None else rows
    out = torch.empty(B, rows, H, D, dtype=like.dtype, device=like.device)
    lse = torch.empty(B, H, rows, dtype=torch.float32, device=like.device)
    if hi > lo:
        # the merge writes a contiguous [B, H, hi - lo] lse; a padded slice
        # takes it through a temporary
        l_dst = lse if rows == hi - lo else torch.empty(B, H, hi - lo, dtype=torch.float32, device=like.device)
        be.merge(parts, out[:, :hi - lo], l_dst)
        if l_dst is not lse:
            lse[:, :, :hi - lo].copy_(l_dst)
    return out, lse


class PeerExchange:
    """Receive buffers of every rank of `group`, mapped into every rank's
    process (CUDA IPC through the library's llmx_ipc_* calls), for the fused
    KV-split exchange: rank s's attention kernel writes each row of its
    partial straight into the buffer of the rank that owns the row
    (llmx_attn_fwd_scatter), so no separate transfer step follows the
    kernel; a one-element all-reduce on the stream then orders every rank's
    writes before the merges.

    Layout of a rank's buffer set: for each source rank s, O as
    [B, slice_rows, H, D] (input dtype), then for each s, lse as
    [B, H, slice_rows] fp32.  Two sets alternate between calls, so a rank's
    next kernel never overwrites rows a slower rank is still merging (its
    next kernel starts only after the next barrier, which that rank enters
    after its merge).  Collective: every rank of the group constructs it with
    the same arguments; close() it on every rank before destroying the group.
    """

    def __init__(self, plan: KVSplitPlan, batch: int, n_heads: int, head_dim: int, dtype: torch.dtype,
                 device, group=None):
        import torch.distributed as dist

        self.plan, self.B, self.H, self.D, self.dtype = plan, batch, n_heads, head_dim, dtype
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if plan.world != self.world:
            raise ValueError("the plan is for a different number of ranks")
        es = torch.tensor([], dtype=dtype).element_size()
        rows = plan.slice_rows
        self.o_bytes = -(-batch * rows * n_heads * head_dim * es // 256) * 256
        self.l_bytes = -(-batch * n_heads * rows * 4 // 256) * 256
        self.set_bytes = self.world * (self.o_bytes + self.l_bytes)
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.check(lib.llmx_ipc_alloc(2 * self.set_bytes, ctypes.byref(ptr), handle))
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.base = []
        self._opened = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.base.append(self._own)
                    continue
                hb = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(h)
                pp = ctypes.c_void_p()
                _lib.check(lib.llmx_ipc_open(hb, ctypes.byref(pp)))
                self.base.append(pp.value)
                self._opened.append(pp.value)
        self.calls = 0

    def o_addr(self, dst: int, src: int, buf: int) -> int:
        return self.base[dst] + buf * self.set_bytes + src * self.o_bytes

    def lse_addr(self, dst: int, src: int, buf: int) -> int:
        return self.base[dst] + buf * self.set_bytes + self.world * self.o_bytes + src * self.l_bytes

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective)."""
        import torch.distributed as dist

        if self._own is None:
            return
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.llmx_ipc_close(ctypes.c_void_p(p))
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            lib.llmx_ipc_free(ctypes.c_void_p(self._own))
        self._own = None


def _fused_kv_split(q, k_chunks, v_chunks, plan, sm_scale, rank, group, alibi_slopes, sliding_window, output,
                    exchange: PeerExchange, timings):
    """kv_split_attention's fused path: one scattered kernel per rank, a
    barrier, the merge of this rank's slice from its own buffer."""
    import torch.distributed as dist

    B, Sq, H, D = q.shape
    dev = q.device
    world = plan.world
    buf = exchange.calls & 1
    exchange.calls += 1
    mine = plan.chunks[rank]
    if mine:
        (a, b), = mine
        r0 = plan.chunk_first_row(a)
        if r0 < Sq:
            p, keep = ops.build_params(q[:, r0:], q[:, r0:], k_chunks[0], v_chunks[0], sm_scale, sliding_window,
                                       alibi_slopes=alibi_slopes, causal=plan.causal, kv_offset=a,
                                       kv_total=plan.kv_len)
            x = _lib.RowScatter()
            x.n_dst, x.slice_rows, x.row_base = world, plan.slice_rows, r0
            for d in range(world):
                x.o[d] = exchange.o_addr(d, rank, buf)
                x.lse[d] = exchange.lse_addr(d, rank, buf)
            lib = _lib.load()
            ws = torch.empty(256, dtype=torch.uint8, device=dev)
            p.workspace, p.workspace_bytes = ws.data_ptr(), 256
            stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
            _lib.check(lib.llmx_attn_fwd_scatter(ctypes.byref(p), ctypes.byref(x), stream))
    _mark(timings, "attention", dev)
    # every rank's scattered writes are fenced system-wide by its kernel; the
    # all-reduce orders them before this rank's merge
    flag = torch.zeros(1, dtype=torch.float32, device=dev)
    dist.all_reduce(flag, group=group)
    _mark(timings, "exchange", dev)
    lo, hi = plan.row_slice(rank)
    rows = plan.slice_rows
    parts = []
    for s in range(world):
        r_lo = max(lo, plan.first_row(s))
        if hi > r_lo:
            parts.append((exchange.o_addr(rank, s, buf) + (r_lo - lo) * H * D * q.element_size(),
                          (rows * H * D, H * D, D),
                          exchange.lse_addr(rank, s, buf) + (r_lo - lo) * 4, (H * rows, rows),
                          r_lo - lo, hi - lo))
    n = rows if output == "replicated" else hi - lo
    out = torch.empty(B, n, H, D, dtype=q.dtype, device=dev)
    lse = torch.empty(B, H, n, dtype=torch.float32, device=dev)
    if hi > lo:
        l_dst = lse if n == hi - lo else torch.empty(B, H, hi - lo, dtype=torch.float32, device=dev)
        CudaOps().merge_raw(parts, out[:, :hi - lo], l_dst)
        if l_dst is not lse:
            lse[:, :, :hi - lo].copy_(l_dst)
    _mark(timings, "merge", dev)
    return out, lse, (lo, hi)


def kv_split_attention(
    q: torch.Tensor,
    k_chunks: Sequence[torch.Tensor],
    v_chunks: Sequence[torch.Tensor],
    plan: KVSplitPlan,
    sm_scale: float,
    *,
    rank: Optional[int] = None,
    group=None,
    alibi_slopes: Optional[torch.Tensor] = None,
    sliding_window: int = -1,
    output: str = "sharded",
    backend=None,
    timings: Optional[list] = None,
    exchange: Optional[PeerExchange] = None,
):
    """Attention of all of `q` ([B, q_len, H, D]) over the keys of every rank
    of `group`, where this rank holds the key chunks `k_chunks` / `v_chunks`
    ([B, n_c, H_kv, D]) at the global positions plan.chunks[rank].

    output="sharded": returns (O [B, hi - lo, H, D], lse [B, H, hi - lo],
    (lo, hi)) for this rank's row slice plan.row_slice(rank);
    output="replicated": returns (O [B, q_len, H, D], lse [B, H, q_len],
    (0, q_len)) on every rank.  Without torch.distributed (or with one rank)
    the plan must have one rank.  `backend` supplies attend / merge (default
    the CUDA kernels); `timings`, if a list, receives (phase, CUDA event)
    marks after the attention, exchange, merge and gather phases.

    exchange: a PeerExchange for this plan and shape selects the fused path
    (the kernel scatters its rows straight into their owners' buffers over
    NVLink; plans with one key range per rank whose first visible row is a
    multiple of 16).  Without it the rows go by NCCL point to point.
    """
    import torch.distributed as dist

    if output not in ("sharded", "replicated"):
        raise ValueError("output must be 'sharded' or 'replicated'")
    multi = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
    world = dist.get_world_size(group) if multi else 1
    if rank is None:
        rank = dist.get_rank(group) if multi else 0
    if plan.world != world:
        raise ValueError(f"the plan is for {plan.world} ranks, the group has {world}")
    B, Sq, H, D = q.shape
    if Sq != plan.q_len:
        raise ValueError("q's length differs from the plan's")
    dev = q.device

    if exchange is not None and multi:
        if any(len(c) > 1 for c in plan.chunks) or any(
                plan.first_row(r) % 16 for r in range(world) if plan.first_row(r) < Sq):
            raise ValueError("the fused exchange takes one key range per rank starting on a 16-row boundary")
        out, lse, (lo, hi) = _fused_kv_split(q, k_chunks, v_chunks, plan, sm_scale, rank, group, alibi_slopes,
                                             sliding_window, output, exchange, timings)
        if output == "sharded":
            return out, lse, (lo, hi)
        return _gather_slices(out, lse, plan, world, group, timings)

    # 1. This rank's partial over its keys, rows [row0, Sq).
    part_o, part_l, row0 = local_partial(q, k_chunks, v_chunks, plan, rank, sm_scale, alibi_slopes=alibi_slopes,
                                         sliding_window=sliding_window, backend=backend)
    _mark(timings, "attention", dev)

    # 2. Row-slice exchange: the rows of my partial in peer p's slice go to p;
    # the sizes come from the plan, so every pair of ranks agrees on them.
    lo, hi = plan.row_slice(rank)
    parts = []
    p2p = []
    for peer in range(world):
        if peer == rank:
            mine = slice_part(part_o, part_l, row0, plan, rank, rank)
            if mine is not None:
                parts.append(mine)
            continue
        out_part = slice_part(part_o, part_l, row0, plan, rank, peer)
        if out_part is not None:
            so, sl = out_part[0], out_part[1]
            so = so if so.is_contiguous() else so.contiguous()
            p2p += [dist.P2POp(dist.isend, so, peer, group), dist.P2POp(dist.isend, sl.contiguous(), peer, group)]
        r_lo = max(lo, plan.first_row(peer))  # the peer holds rows [r_lo, hi) of my slice
        if hi > r_lo:
            ro = torch.empty(B, hi - r_lo, H, D, dtype=q.dtype, device=dev)
            rl = torch.empty(B, H, hi - r_lo, dtype=torch.float32, device=dev)
            p2p += [dist.P2POp(dist.irecv, ro, peer, group), dist.P2POp(dist.irecv, rl, peer, group)]
            parts.append((ro, rl, r_lo - lo, hi - lo))
    if p2p:
        for req in dist.batch_isend_irecv(p2p):
            req.wait()
    _mark(timings, "exchange", dev)

    # 3. Merge of my slice (padded to slice_rows for the all-gather).
    out, lse = merge_slice(parts, plan, rank, q, rows=plan.slice_rows if output == "replicated" else None,
                           backend=backend)
    _mark(timings, "merge", dev)
    if output == "sharded":
        return out, lse, (lo, hi)

    # 4. All-gather of the slices.
    return _gather_slices(out, lse, plan, world, group, timings, multi)


def _gather_slices(out, lse, plan, world, group, timings, multi=True):
    """All-gather of every rank's slice (each padded to slice_rows) into the
    whole output on every rank."""
    import torch.distributed as dist

    B, rows, H, D = out.shape
    Sq = plan.q_len
    dev = out.device
    if multi:
        # concatenated along the batch axis (the layout every backend takes)
        go = torch.empty((world * B,) + tuple(out.shape[1:]), dtype=out.dtype, device=dev)
        gl = torch.empty((world * B,) + tuple(lse.shape[1:]), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(go, out, group=group)
        dist.all_gather_into_tensor(gl, lse, group=group)
        go, gl = go.view((world,) + tuple(out.shape)), gl.view((world,) + tuple(lse.shape))
    else:
        go, gl = out.unsqueeze(0), lse.unsqueeze(0)
    full = go.permute(1, 0, 2, 3, 4).reshape(B, world * rows, H, D)[:, :Sq]
    full_l = gl.permute(1, 2, 0, 3).reshape(B, H, world * rows)[:, :, :Sq].contiguous()
    _mark(timings, "gather", dev)
    return full, full_l, (0, Sq)
