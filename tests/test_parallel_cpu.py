"""Multi-GPU host logic on CPU: unit / head / key sharding, the KV-split plan,
and the KV-split exchange run by 2 and 4 `gloo` ranks.  The attention
partials and the merge come from the CPU oracle (the checker, standing in for
the kernels); the code under test is llmx_b200.parallel's partitioning, its
row-restricted partials and its point-to-point row-slice exchange."""
import os

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from llmx_b200 import parallel
from llmx_b200.workloads import visible_pairs


@pytest.mark.parametrize("B,H,world", [(8, 32, 1), (8, 32, 2), (64, 32, 8), (1, 32, 8), (3, 5, 4), (1, 1, 2)])
def test_shard_units_cover_once_and_balance(B, H, world):
    seen = []
    sizes = []
    for r in range(world):
        s, e = parallel.shard_units(B, H, world, r)
        seen.extend(range(s, e))
        sizes.append(e - s)
    assert seen == list(range(B * H))
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("S,world", [(32768, 2), (32768, 4), (32768, 8), (1000, 3), (100, 8)])
def test_zigzag_chunks_cover_once_and_balance_causal_work(S, world):
    covered = []
    work = []
    for r in range(world):
        ch = parallel.zigzag_chunks(S, world, r)
        w = 0
        for a, b in ch:
            covered.extend(range(a, b))
            # visible causal pairs of all S queries over keys [a, b)
            w += sum(max(0, S - max(a, j)) for j in range(a, b)) if S <= 4096 else (b - a) * (S - (a + b - 1) / 2)
        work.append(w)
    assert sorted(covered) == list(range(S))
    if S >= 32768:
        assert max(work) / min(work) < 1.02


@pytest.mark.parametrize("S,world", [(32768, 2), (32768, 4), (32768, 8), (131072, 8), (1000, 3), (100, 8)])
def test_causal_key_range_covers_once_and_balances_causal_work(S, world):
    ranges = [parallel.causal_key_range(S, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == S
    for (a0, b0), (a1, b1) in zip(ranges, ranges[1:]):
        assert a0 <= b0 == a1 <= b1
    # visible causal pairs of all S queries over keys [a, b): sum of S - j
    work = [(b - a) * S - (b * (b - 1) - a * (a - 1)) / 2 for a, b in ranges]
    assert sum(work) == S * (S + 1) / 2
    if S >= 32768:
        assert max(work) / min(work) < 1.01


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_kv_split_ranges_cover_every_key_once(world):
    S = 32768
    covered = sorted(j for r in range(world) for a, b in parallel.kv_split_ranges(S, world, r) for j in range(a, b))
    assert covered == list(range(S))


@pytest.mark.parametrize("S,world", [(33, 3), (48, 3), (100, 8), (128, 8), (20, 2), (16, 2), (32, 2)])
def test_causal_key_range_gives_every_rank_a_block_when_possible(S, world):
    ranges = [parallel.causal_key_range(S, world, r) for r in range(world)]
    covered = sorted(j for a, b in ranges for j in range(a, b))
    assert covered == list(range(S))
    if S >= world * 16:
        assert all(b - a >= 16 for a, b in ranges), ranges
    else:
        # too short for a block per rank: the first ceil(S / 16) ranks take one each
        assert sum(1 for a, b in ranges if b > a) == -(-S // 16)


def _model_cost_bruteforce(a, b, S, item_rows=256, block=128, item_cost=1.5):
    # item by item, row by row: the item's block count is that of its last row
    total, r = 0.0, a
    while r < S:
        last = min(S - 1, r + item_rows - 1)
        seen = min(b, last + 1) - a
        if seen > 0:
            total += item_cost + -(-seen // block)
        r += item_rows
    return total


@pytest.mark.parametrize("a,b,S", [(0, 32768, 32768), (0, 100, 1000), (128, 1000, 1000), (384, 1024, 4096),
                                   (16384, 32768, 32768), (5, 5, 64)])
def test_key_range_cost_matches_item_by_item_count(a, b, S):
    assert parallel.key_range_cost(a, b, S, S) == _model_cost_bruteforce(a, b, S)


@pytest.mark.parametrize("S,world", [(32768, 2), (32768, 4), (32768, 8), (131072, 8), (1000, 3), (4096, 8),
                                     (300, 3), (100, 8), (20, 2), (128, 4)])
def test_balanced_key_ranges_cover_once_aligned_and_balanced(S, world):
    ranges = parallel.balanced_key_ranges(S, world)
    assert len(ranges) == world
    covered = sorted(j for a, b in ranges for j in range(a, b))
    assert covered == list(range(S))
    nonempty = [(a, b) for a, b in ranges if b > a]
    for a, b in nonempty:
        assert a % 128 == 0 and (b % 128 == 0 or b == S)
    assert len(nonempty) == min(world, -(-S // 128))
    assert ranges[:len(nonempty)] == nonempty  # empty ranges only at the end
    if S >= 32768:
        cost = [parallel.key_range_cost(a, b, S, S) for a, b in ranges]
        pairs = [parallel.causal_key_range(S, world, r) for r in range(world)]
        pair_cost = [parallel.key_range_cost(a, b, S, S) for a, b in pairs]
        # no worse than the pair-balanced split on the kernel model, and
        # within a few blocks per rank of the mean
        assert max(cost) <= max(pair_cost) + 1e-9
        assert max(cost) - sum(cost) / world < 0.03 * sum(cost) / world


def test_contiguous_plan_balance_choice():
    S, world = 32768, 8
    kern = parallel.KVSplitPlan.contiguous(S, world)
    pairs = parallel.KVSplitPlan.contiguous(S, world, balance="pairs")
    assert [c[0] for c in kern.chunks] == parallel.balanced_key_ranges(S, world)
    assert [c[0] for c in pairs.chunks] == [parallel.causal_key_range(S, world, r) for r in range(world)]
    with pytest.raises(ValueError):
        parallel.KVSplitPlan.contiguous(S, world, balance="rows")
    # without the causal mask both give even ranges
    assert parallel.KVSplitPlan.contiguous(S, world, causal=False).chunks == \
        parallel.KVSplitPlan.contiguous(S, world, causal=False, balance="pairs").chunks


@pytest.mark.parametrize("weights,heads,world,align", [
    ([565 ** 2, 953 ** 2, 721 ** 2, 968 ** 2], 16, 8, 1),   # padded prefill: visible pairs per sequence
    ([271, 4010, 1500, 2048, 300, 999], 32, 4, 4),          # decode key lengths, GQA groups of 4
    ([5, 5, 5, 5], 8, 3, 2),
    ([1, 0, 7], 2, 8, 1),                                    # more ranks than units: empty ranges
    ([0, 0], 4, 2, 1),                                       # no work at all: even split
])
def test_shard_units_weighted_covers_once_aligned_and_balanced(weights, heads, world, align):
    ranges = [parallel.shard_units_weighted(weights, heads, world, r, align=align) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == len(weights) * heads
    for (a0, b0), (a1, b1) in zip(ranges, ranges[1:]):
        assert a0 <= b0 == a1 <= b1
    for a, b in ranges:
        assert a % align == 0 and b % align == 0
    total = sum(weights) * heads
    if total > 0:
        load = [sum(weights[u // heads] for u in range(a, b)) for a, b in ranges]
        heaviest = max(weights) * align
        # every rank within one granule of its equal share
        assert all(abs(x - total / world) <= heaviest for x in load), load


@pytest.mark.parametrize("batch,heads,world,group,want", [
    (4, 16, 2, 1, 16), (4, 16, 4, 1, 16), (4, 16, 8, 1, 8), (64, 32, 8, 1, 32), (1, 32, 8, 4, 4),
    (2, 12, 8, 3, 3), (1, 8, 16, 1, 1), (1, 12, 2, 1, 6)])
def test_launch_granule(batch, heads, world, group, want):
    g = parallel.launch_granule(batch, heads, world, group)
    assert g == want
    assert heads % g == 0 and g % group == 0
    # whole-granule ranges give every rank at most one launch per run of sequences
    w = [1.0 + b for b in range(batch)]
    for r in range(world):
        a, b = parallel.shard_units_weighted(w, heads, world, r, align=g)
        if g == heads:
            assert len(parallel.unit_runs(a, b, heads)) <= 1


def test_shard_units_weighted_equal_weights_match_shard_units():
    for world in (1, 2, 4, 8):  # an even split: the same ranges
        assert [parallel.shard_units_weighted([1.0] * 8, 32, world, r) for r in range(world)] == \
            [parallel.shard_units(8, 32, world, r) for r in range(world)]
    sizes = [b - a for a, b in (parallel.shard_units_weighted([1.0] * 8, 32, 3, r) for r in range(3))]
    assert sum(sizes) == 256 and max(sizes) - min(sizes) <= 1  # otherwise sizes within one unit
    with pytest.raises(ValueError):
        parallel.shard_units_weighted([1, 2], 6, 2, 0, align=4)


@pytest.mark.parametrize("start,end,heads", [(0, 256, 32), (32, 64, 32), (5, 70, 32), (3, 9, 4), (0, 1, 1),
                                             (10, 10, 4)])
def test_unit_runs_cover_the_range(start, end, heads):
    runs = parallel.unit_runs(start, end, heads)
    assert len(runs) <= 3
    units = [b * heads + h for b0, b1, h0, h1 in runs for b in range(b0, b1) for h in range(h0, h1)]
    assert units == list(range(start, end))


@pytest.mark.parametrize("H,world,group", [(32, 8, 1), (32, 2, 1), (32, 8, 4), (12, 5, 3), (32, 3, 8)])
def test_head_range_deals_whole_groups(H, world, group):
    rs = [parallel.head_range(H, world, r, group) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == H
    for (a0, b0), (a1, b1) in zip(rs, rs[1:]):
        assert b0 == a1
    assert all(a % group == 0 and b % group == 0 for a, b in rs)


@pytest.mark.parametrize("make", ["contiguous", "zigzag"])
@pytest.mark.parametrize("S,world", [(32768, 8), (32768, 2), (300, 2), (20, 2), (333, 4), (20, 3)])
def test_kv_split_plan_rows_and_keys(make, S, world):
    plan = getattr(parallel.KVSplitPlan, make)(S, world)
    keys = sorted(j for r in range(world) for a, b in plan.chunks[r] for j in range(a, b))
    assert keys == list(range(S))
    rows = sorted(i for r in range(world) for i in range(*plan.row_slice(r)))
    assert rows == list(range(S))
    for r in range(world):
        ks = [a for a, b in plan.chunks[r] if b > a]
        # causal, q_len == kv_len: row i sees key a iff i >= a
        assert plan.first_row(r) == (min(ks) if ks else S)


def _partials(q, k, v, chunks, alibi, S):
    outs, lses = [], []
    for a, b in chunks:
        o, l = oracle.attention_ref(q[0], k[0, a:b], v[0, a:b], alibi=alibi, return_lse=True, kv_offset=a,
                                    kv_total=S)
        outs.append(o.unsqueeze(0))
        lses.append(l.unsqueeze(0))
    return outs, lses


def test_merge_of_causal_key_ranges_equals_full_attention():
    g = torch.Generator().manual_seed(2)
    S, H, D = 333, 2, 32
    q, k, v = (torch.randn(1, S, H, D, generator=g) for _ in range(3))
    a = oracle.alibi_slopes(H)
    full, lfull = oracle.attention_ref(q[0], k[0], v[0], alibi=a, return_lse=True)
    chunks = [parallel.causal_key_range(S, 4, r) for r in range(4)]
    outs, lses = _partials(q, k, v, chunks, a, S)
    out, lse = oracle.merge_partials(outs, lses)
    torch.testing.assert_close(out[0], full, atol=2e-6, rtol=0)
    torch.testing.assert_close(lse[0], lfull, atol=2e-6, rtol=0)


class OracleOps:
    """CPU stand-in for the kernels (parallel.CudaOps): the oracle computes
    each chunk's partial and the merge, so the test exercises the plan, the
    row restriction and the exchange of llmx_b200.parallel."""

    def attend(self, o, lse, q, k, v, sm_scale, *, alibi_slopes, causal, sliding_window, kv_offset, kv_total):
        for b in range(q.shape[0]):
            ob, lb = oracle.attention_ref(q[b], k[b], v[b], sm_scale=sm_scale, alibi=alibi_slopes, causal=causal,
                                          sliding_window=sliding_window, return_lse=True, kv_offset=kv_offset,
                                          kv_total=kv_total)
            o[b] = ob
            lse[b] = lb

    def merge(self, parts, out, lse_out):
        B, S, H, D = out.shape
        O, L = oracle.merge_row_parts(parts, B, S, H, D)
        out.copy_(O.to(out.dtype))
        if lse_out is not None:
            lse_out.copy_(L)


def _split_inputs(S, B=1, H=2, D=16, seed=1):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(B, S, H, D, generator=g) for _ in range(3))


def _kv_rank(rank, world, port, S, make, output, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    B = 2 if S == 333 else 1
    q, k, v = _split_inputs(S, B=B)
    plan = getattr(parallel.KVSplitPlan, make)(S, world)
    mine = plan.chunks[rank]
    out, lse, (lo, hi) = parallel.kv_split_attention(
        q, [k[:, a:b] for a, b in mine], [v[:, a:b] for a, b in mine], plan, 16 ** -0.5,
        alibi_slopes=oracle.alibi_slopes(2), output=output, backend=OracleOps())
    torch.save({"out": out, "lse": lse, "rows": (lo, hi)}, f"{result_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,S,make,output", [
    (2, 20, "contiguous", "sharded"),    # short: rank 1 holds no keys
    (2, 300, "zigzag", "sharded"),       # rank 0 keeps one chunk, rank 1 two
    (2, 300, "contiguous", "replicated"),
    (4, 333, "contiguous", "sharded"),   # batch 2
    (4, 333, "zigzag", "replicated"),
    (4, 40, "contiguous", "replicated"),  # ranks 3 has no keys, some slices empty
])
def test_kv_split_exchange_over_gloo_ranks(tmp_path, world, S, make, output):
    path = str(tmp_path / "kv")
    port = 29500 + (os.getpid() * 7 + world * 31 + S) % 2000
    mp.spawn(_kv_rank, args=(world, port, S, make, output, path), nprocs=world, join=True)
    B = 2 if S == 333 else 1
    q, k, v = _split_inputs(S, B=B)
    a = oracle.alibi_slopes(2)
    for r in range(world):
        res = torch.load(f"{path}.{r}")
        lo, hi = res["rows"]
        if output == "replicated":
            assert (lo, hi) == (0, S)
        for b in range(B):
            full, lfull = oracle.attention_ref(q[b], k[b], v[b], alibi=a, return_lse=True)
            torch.testing.assert_close(res["out"][b], full[lo:hi], atol=2e-6, rtol=0)
            torch.testing.assert_close(res["lse"][b], lfull[:, lo:hi], atol=2e-6, rtol=0)
