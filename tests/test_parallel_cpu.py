"""Multi-GPU host logic on CPU: unit sharding, zig-zag key chunks and the
exact log-sum-exp merge, including the cross-rank merge run by two `gloo`
ranks.  Partials come from the CPU oracle (the checker); the code under test
is llmx_b200.parallel's partitioning and merge."""
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


def test_merge_of_causal_key_ranges_equals_full_attention():
    g = torch.Generator().manual_seed(2)
    S, H, D = 333, 2, 32
    q, k, v = (torch.randn(1, S, H, D, generator=g) for _ in range(3))
    a = oracle.alibi_slopes(H)
    full, lfull = oracle.attention_ref(q[0], k[0], v[0], alibi=a, return_lse=True)
    chunks = [parallel.causal_key_range(S, 4, r) for r in range(4)]
    outs, lses = _partials(q, k, v, chunks, a, S)
    out, lse = parallel.merge_partials(outs, lses)
    torch.testing.assert_close(out[0], full, atol=2e-6, rtol=0)
    torch.testing.assert_close(lse[0], lfull, atol=2e-6, rtol=0)


def _partials(q, k, v, chunks, alibi, S):
    outs, lses = [], []
    for a, b in chunks:
        o, l = oracle.attention_ref(q[0], k[0, a:b], v[0, a:b], alibi=alibi, return_lse=True, kv_offset=a,
                                    kv_total=S)
        outs.append(o.unsqueeze(0))
        lses.append(l.unsqueeze(0))
    return outs, lses


def test_merge_partials_equals_full_attention():
    g = torch.Generator().manual_seed(0)
    S, H, D = 300, 2, 32
    q, k, v = (torch.randn(1, S, H, D, generator=g) for _ in range(3))
    a = oracle.alibi_slopes(H)
    full, lfull = oracle.attention_ref(q[0], k[0], v[0], alibi=a, return_lse=True)
    chunks = [c for r in range(3) for c in parallel.zigzag_chunks(S, 3, r, align=16)]
    outs, lses = _partials(q, k, v, chunks, a, S)
    out, lse = parallel.merge_partials(outs, lses)
    torch.testing.assert_close(out[0], full, atol=2e-6, rtol=0)
    torch.testing.assert_close(lse[0], lfull, atol=2e-6, rtol=0)


def _rank(rank, world, port, S, H, D, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, S, H, D, generator=g) for _ in range(3))
    a = oracle.alibi_slopes(H)
    chunks = parallel.zigzag_chunks(S, world, rank, align=32)
    outs, lses = _partials(q, k, v, chunks, a, S)
    out, lse = parallel.merge_partials(outs, lses)
    out, lse = parallel.merge_across_ranks(out, lse)
    if rank == 0:
        torch.save({"out": out, "lse": lse}, result_path)
    dist.barrier()
    dist.destroy_process_group()


def test_merge_across_two_gloo_ranks(tmp_path):
    S, H, D = 256, 2, 16
    path = str(tmp_path / "merged.pt")
    port = 29500 + os.getpid() % 1000
    mp.spawn(_rank, args=(2, port, S, H, D, path), nprocs=2, join=True)
    res = torch.load(path)
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(1, S, H, D, generator=g) for _ in range(3))
    full, lfull = oracle.attention_ref(q[0], k[0], v[0], alibi=oracle.alibi_slopes(H), return_lse=True)
    torch.testing.assert_close(res["out"][0], full, atol=2e-6, rtol=0)
    torch.testing.assert_close(res["lse"][0], lfull, atol=2e-6, rtol=0)
