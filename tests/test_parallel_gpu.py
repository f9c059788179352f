"""Key shards, unit / head shards and the KV-split long-context path on the GPU.

* every kernel family with kv_offset / kv_total (a shard of a sequence's keys
  at its global positions) against the oracle evaluated on the same keys;
* the KV split of 2, 4 and 8 virtual ranks run on one GPU (each rank's
  row-restricted partial, the row slices each rank would receive, the merge
  kernel), every output row against the unsplit kernel and the fp32 oracle;
* the merge kernel against the oracle's merge (row ranges, strided views,
  rows a part does not cover holding NaN);
* unit and head shards against the unsplit call (bit-identical);
* the row-scattered kernel output (llmx_attn_fwd_scatter) of 2, 4 and 8
  virtual ranks into per-destination buffers on one GPU, merged per slice,
  against the unsplit kernel;
* with two or more GPUs, the real 2-rank split: NCCL point to point (both
  plans, both output forms, the short sequences where a rank holds one chunk
  or none) and the fused exchange (the kernel writing into the peer's
  buffer through CUDA IPC).
Tolerances: see gpu_helpers.
"""
import os

import pytest
import torch
import torch.multiprocessing as mp

import llmx_b200
import oracle
from gpu_helpers import assert_close, needs_cuda
from llmx_b200 import parallel

pytestmark = [pytest.mark.gpu, needs_cuda]


def rand(*shape, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


@pytest.mark.parametrize("algo", ["simt", "tcgen05", "decode"])
@pytest.mark.parametrize("window", [-1, 200])
def test_key_shard_geometry(algo, window):
    S, H, D = 700, 4, 128
    a0, a1 = 256, 640  # this shard holds global keys [256, 640) of 700
    q = rand(1, S if algo != "decode" else 1, H, D)
    k = rand(1, S, H, D, seed=1)
    v = rand(1, S, H, D, seed=2)
    slopes = oracle.alibi_slopes(H)
    qd, kd, vd = q.cuda(), k[:, a0:a1].contiguous().cuda(), v[:, a0:a1].contiguous().cuda()
    out = torch.full_like(qd, float("nan"))
    lse = torch.empty(1, H, q.shape[1], device="cuda")
    llmx_b200.single_mha_attention_half(out, qd, kd, vd, D ** -0.5, window, alibi_slopes=slopes.cuda(), lse=lse,
                                        algo=algo, kv_offset=a0, kv_total=S)
    torch.cuda.synchronize()
    # the single decode row is the last query of the sequence
    ql = q.shape[1]
    ref, lref = oracle.attention_ref(q[0].float(), k[0, a0:a1].float(), v[0, a0:a1].float(), alibi=slopes,
                                     sliding_window=window, return_lse=True, kv_offset=a0, kv_total=S)
    assert_close(out[0], ref, torch.bfloat16, f"shard/{algo}")
    fin = torch.isfinite(lref)
    assert torch.equal(torch.isfinite(lse[0].cpu()), fin)
    torch.testing.assert_close(lse[0].cpu()[fin], lref[fin], atol=2e-3, rtol=0)
    assert ql >= 1


def _virtual_split(q, k, v, plan, slopes, sm_scale):
    """Runs every virtual rank's partial, then every rank's slice merge, on
    this GPU; returns the full output and lse assembled from the slices."""
    B, S, H, D = q.shape
    partials = []
    for r in range(plan.world):
        kc = [k[:, a:b] for a, b in plan.chunks[r]]
        vc = [v[:, a:b] for a, b in plan.chunks[r]]
        partials.append(parallel.local_partial(q, kc, vc, plan, r, sm_scale, alibi_slopes=slopes))
    out = torch.empty_like(q)
    lse = torch.empty(B, H, S, device=q.device)
    for dst in range(plan.world):
        parts = [p for p in (parallel.slice_part(o, l, r0, plan, src, dst)
                             for src, (o, l, r0) in enumerate(partials)) if p is not None]
        lo, hi = plan.row_slice(dst)
        o, l = parallel.merge_slice(parts, plan, dst, q)
        out[:, lo:hi] = o
        lse[:, :, lo:hi] = l
    return out, lse


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("make", ["contiguous", "zigzag"])
def test_kv_split_virtual_ranks_every_row(world, make):
    S, H, D = 4096, 4, 128
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    full = torch.empty_like(q)
    lfull = torch.empty(1, H, S, device="cuda")
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=slopes, lse=lfull)
    plan = getattr(parallel.KVSplitPlan, make)(S, world)
    out, lse = _virtual_split(q, k, v, plan, slopes, D ** -0.5)
    torch.cuda.synchronize()
    assert (out.float() - full.float()).abs().max().item() <= 2e-2
    torch.testing.assert_close(lse, lfull, atol=1e-3, rtol=0)
    ref, lref = oracle.attention_ref_chunked(q, k, v, alibi=slopes)
    assert_close(out, ref, torch.bfloat16, f"kv split {make}/{world}")
    torch.testing.assert_close(lse, lref, atol=2e-3, rtol=0)


def test_kv_split_one_rank_api():
    S, H, D = 2048, 4, 128
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    full = torch.empty_like(q)
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=slopes)
    plan = parallel.KVSplitPlan.zigzag(S, 1)  # two chunks on the one rank: the local merge
    for output in ("sharded", "replicated"):
        out, lse, rows = parallel.kv_split_attention(q, [k[:, a:b] for a, b in plan.chunks[0]],
                                                     [v[:, a:b] for a, b in plan.chunks[0]], plan, D ** -0.5,
                                                     alibi_slopes=slopes, output=output)
        torch.cuda.synchronize()
        assert rows == (0, S)
        assert (out.float() - full.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n_parts,S,H,D", [(1, 96, 3, 64), (3, 300, 2, 128), (8, 257, 2, 128), (16, 64, 1, 256),
                                           (2, 40, 5, 8), (0, 33, 2, 64)])
def test_merge_kernel_matches_oracle(dtype, n_parts, S, H, D):
    g = torch.Generator().manual_seed(n_parts * 7 + S)
    B = 2
    parts, cpu_parts = [], []
    for c in range(n_parts):
        lo = int(torch.randint(0, S // 2, (1,), generator=g))
        hi = int(torch.randint(lo, S + 1, (1,), generator=g)) if c else S
        n = hi - lo
        # a strided view: every other row of a larger buffer
        big = torch.randn(B, 2 * n + 1, H, D, generator=g).to(dtype)
        lse = torch.randn(B, H, n, generator=g) * 3
        if n > 2:
            lse[:, :, 1] = float("-inf")  # a row this part never saw...
            big[:, 2] = float("nan")       # ...whose O must not be read
        o_dev = big.cuda()[:, ::2][:, :n]  # a strided view on the device
        parts.append((o_dev, lse.cuda(), lo, hi))
        cpu_parts.append((big[:, ::2][:, :n].float().nan_to_num(0.0), lse, lo, hi))
    out = torch.full((B, S, H, D), float("nan"), dtype=dtype, device="cuda")
    lse_out = torch.empty(B, H, S, device="cuda")
    parallel.CudaOps().merge(parts, out, lse_out)
    torch.cuda.synchronize()
    ref, lref = oracle.merge_row_parts(cpu_parts, B, S, H, D)
    assert torch.isfinite(out.float()).all()
    assert (out.float().cpu() - ref).abs().max().item() <= 2e-2
    fin = torch.isfinite(lref)
    assert torch.equal(torch.isfinite(lse_out.cpu()), fin)
    torch.testing.assert_close(lse_out.cpu()[fin], lref[fin], atol=1e-4, rtol=0)


@pytest.mark.parametrize("world", [3, 8])
def test_weighted_unit_shards_of_a_padded_batch_match_the_whole_call(world):
    """Padded, non-causal fp16 prefill with ALiBi (the shape of the padded
    workload, smaller): units dealt by visible pairs, each shard run with its
    own sequences' lengths, bit-identical to the whole call."""
    B, S, H, D = 4, 384, 4, 64
    lens = [200, 384, 131, 300]
    q, k, v = (rand(B, S, H, D, seed=20 + s, dtype=torch.float16).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    ql = torch.tensor(lens, dtype=torch.int32, device="cuda")
    kw = dict(alibi_slopes=slopes, causal=False, q_lens=ql, kv_lens=ql)
    full = torch.empty_like(q)
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, **kw)
    out = torch.full_like(q, float("nan"))
    weights = [n * n for n in lens]
    for r in range(world):
        s0, s1 = parallel.shard_units_weighted(weights, H, world, r)
        parallel.run_units(out, q, k, v, s0, s1, D ** -0.5, **kw)
    torch.cuda.synchronize()
    assert torch.equal(out, full)


def test_weighted_unit_shards_of_a_decode_batch_match_the_whole_call():
    """Batched decode with unequal key lengths and GQA: units dealt by key
    length in whole groups; each shard's split-KV plan may differ from the
    whole call's, so the check is the parity tolerance (and the oracle)."""
    B, S, H, Hkv, D = 6, 1024, 8, 2, 128
    lens = [1024, 37, 500, 777, 1, 256]
    q = rand(B, 1, H, D, seed=31, dtype=torch.bfloat16).cuda()
    k, v = (rand(B, S, Hkv, D, seed=32 + s, dtype=torch.bfloat16).cuda() for s in range(2))
    slopes = oracle.alibi_slopes(H).cuda()
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    kw = dict(alibi_slopes=slopes, kv_lens=kl)
    full = torch.empty_like(q)
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, **kw)
    out = torch.full_like(q, float("nan"))
    for r in range(3):
        s0, s1 = parallel.shard_units_weighted(lens, H, 3, r, align=H // Hkv)
        parallel.run_units(out, q, k, v, s0, s1, D ** -0.5, **kw)
    torch.cuda.synchronize()
    assert_close(out, full, torch.bfloat16, "decode unit shards vs whole call")
    for b in (0, 1, 4):
        ref = oracle.attention_ref(q[b].cpu(), k[b, :lens[b]].cpu(), v[b, :lens[b]].cpu(), sm_scale=D ** -0.5,
                                   alibi=slopes.cpu())
        assert_close(out[b], ref, torch.bfloat16, f"decode sequence {b}")


def test_merge_kernel_full_slice():
    """One rank's row slice of the 32768-token split at 4 GPUs: four bf16
    partials of 8192 rows x 32 heads x 128 (one covering only its later
    rows), merged by the kernel against the same merge in fp32 torch on the
    GPU (the formula the oracle's merge, pinned above, states)."""
    B, S, H, D = 1, 8192, 32, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    ranges = [(0, S), (0, S), (1000, S), (0, S)]
    parts = []
    for lo, hi in ranges:
        o = torch.randn(B, hi - lo, H, D, generator=g, device="cuda").to(torch.bfloat16)
        lse = torch.randn(B, H, hi - lo, generator=g, device="cuda") * 4
        lse[:, :, ::97] = float("-inf")
        parts.append((o, lse, lo, hi))
    out = torch.empty(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    lse_out = torch.empty(B, H, S, device="cuda")
    parallel.CudaOps().merge(parts, out, lse_out)
    # fp32 reference: every part padded to all rows with lse = -inf
    L = torch.full((len(parts), B, H, S), float("-inf"), device="cuda")
    O = torch.zeros(len(parts), B, S, H, D, device="cuda")
    for c, (o, lse, lo, hi) in enumerate(parts):
        L[c, :, :, lo:hi] = lse
        O[c, :, lo:hi] = o.float()
    m = L.max(dim=0).values
    w = torch.where(L == float("-inf"), torch.zeros_like(L), torch.exp(L - m))
    W = w.sum(dim=0)
    ref = (w.permute(0, 1, 3, 2).unsqueeze(-1) * O).sum(dim=0) / W.permute(0, 2, 1).unsqueeze(-1).clamp_min(1e-30)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 2e-2
    fin = W > 0
    torch.testing.assert_close(lse_out[fin], (m + torch.log(W))[fin], atol=1e-4, rtol=1e-6)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_unit_and_head_shards_match_the_whole_call(world):
    B, S, H, D = 3, 512, 8, 128
    q, k, v = (rand(B, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    full = torch.empty_like(q)
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=slopes)
    out = torch.full_like(q, float("nan"))
    for r in range(world):
        s, e = parallel.shard_units(B, H, world, r)
        parallel.run_units(out, q, k, v, s, e, D ** -0.5, alibi_slopes=slopes)
    torch.cuda.synchronize()
    assert torch.equal(out, full)
    out2 = torch.full_like(q, float("nan"))
    for r in range(world):
        h0, h1 = parallel.head_range(H, world, r)
        llmx_b200.single_mha_attention_half(out2[:, :, h0:h1], q[:, :, h0:h1], k[:, :, h0:h1], v[:, :, h0:h1],
                                            D ** -0.5, alibi_slopes=slopes[h0:h1])
    torch.cuda.synchronize()
    assert torch.equal(out2, full)


def _nccl_rank(rank, world, port, S, H, D, path, make, output):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    plan = getattr(parallel.KVSplitPlan, make)(S, world)
    mine = plan.chunks[rank]
    out, lse, rows = parallel.kv_split_attention(q, [k[:, a:b] for a, b in mine], [v[:, a:b] for a, b in mine],
                                                 plan, D ** -0.5, alibi_slopes=slopes, output=output)
    torch.cuda.synchronize()
    torch.save({"out": out.cpu(), "lse": lse.cpu(), "rows": rows}, f"{path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("S,make,output", [(8192, "zigzag", "sharded"), (8192, "contiguous", "replicated"),
                                           (20, "contiguous", "sharded"), (300, "zigzag", "replicated")])
def test_kv_split_two_gpus_nccl(tmp_path, S, make, output):
    H, D = 4, 128
    path = str(tmp_path / "split")
    port = 29600 + (os.getpid() * 7 + S + len(make) + len(output)) % 1000
    mp.spawn(_nccl_rank, args=(2, port, S, H, D, path, make, output), nprocs=2, join=True)
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    full = torch.empty_like(q)
    lse = torch.empty(1, H, S, device="cuda")
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=oracle.alibi_slopes(H).cuda(),
                                        lse=lse)
    torch.cuda.synchronize()
    for r in range(2):
        res = torch.load(f"{path}.{r}")
        lo, hi = res["rows"]
        assert (res["out"].float() - full[:, lo:hi].float().cpu()).abs().max().item() <= 2e-2
        torch.testing.assert_close(res["lse"], lse[:, :, lo:hi].cpu(), atol=1e-3, rtol=0)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_scattered_kernel_output_virtual_ranks(world):
    import ctypes

    from llmx_b200 import _lib, ops

    S, H, D = 4096, 4, 128
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    full = torch.empty_like(q)
    lfull = torch.empty(1, H, S, device="cuda")
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=slopes, lse=lfull)
    plan = parallel.KVSplitPlan.contiguous(S, world)
    rows = plan.slice_rows
    # recv[dst][src]: what source src's kernel writes for destination dst
    recv_o = [[torch.full((1, rows, H, D), float("nan"), dtype=q.dtype, device="cuda") for _ in range(world)]
              for _ in range(world)]
    recv_l = [[torch.full((1, H, rows), float("nan"), device="cuda") for _ in range(world)] for _ in range(world)]
    lib = _lib.load()
    for src in range(world):
        if not plan.chunks[src]:
            continue
        (a, b), = plan.chunks[src]
        r0 = plan.chunk_first_row(a)
        p, keep = ops.build_params(q[:, r0:], q[:, r0:], k[:, a:b], v[:, a:b], D ** -0.5, alibi_slopes=slopes,
                                   kv_offset=a, kv_total=S)
        x = _lib.RowScatter()
        x.n_dst, x.slice_rows, x.row_base = world, rows, r0
        for d in range(world):
            x.o[d] = recv_o[d][src].data_ptr()
            x.lse[d] = recv_l[d][src].data_ptr()
        _lib.check(lib.llmx_attn_fwd_scatter(ctypes.byref(p), ctypes.byref(x),
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    out = torch.empty_like(q)
    for dst in range(world):
        lo, hi = plan.row_slice(dst)
        parts = []
        for src in range(world):
            r_lo = max(lo, plan.first_row(src))
            if hi > r_lo:
                parts.append((recv_o[dst][src][:, r_lo - lo:hi - lo], recv_l[dst][src][:, :, r_lo - lo:hi - lo],
                              r_lo - lo, hi - lo))
        o, l = parallel.merge_slice(parts, plan, dst, q)
        out[:, lo:hi] = o
        torch.testing.assert_close(l, lfull[:, :, lo:hi], atol=1e-3, rtol=1e-6)
    torch.cuda.synchronize()
    assert (out.float() - full.float()).abs().max().item() <= 2e-2


def _fused_rank(rank, world, port, S, H, D, path, output):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    plan = parallel.KVSplitPlan.contiguous(S, world)
    ex = parallel.PeerExchange(plan, 1, H, D, q.dtype, q.device)
    mine = plan.chunks[rank]
    res = []
    for _ in range(3):  # both buffer sets, then the first again
        out, lse, rows = parallel.kv_split_attention(q, [k[:, a:b] for a, b in mine], [v[:, a:b] for a, b in mine],
                                                     plan, D ** -0.5, alibi_slopes=slopes, output=output, exchange=ex)
        res.append((out.cpu(), lse.cpu(), rows))
    torch.cuda.synchronize()
    ex.close()
    torch.save(res, f"{path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("output", ["sharded", "replicated"])
def test_kv_split_two_gpus_fused_exchange(tmp_path, output):
    S, H, D = 8192, 4, 128
    path = str(tmp_path / "fused")
    port = 29700 + (os.getpid() * 7 + len(output)) % 1000
    mp.spawn(_fused_rank, args=(2, port, S, H, D, path, output), nprocs=2, join=True)
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    full = torch.empty_like(q)
    lse = torch.empty(1, H, S, device="cuda")
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=oracle.alibi_slopes(H).cuda(),
                                        lse=lse)
    torch.cuda.synchronize()
    for r in range(2):
        for out, l, (lo, hi) in torch.load(f"{path}.{r}"):
            assert (out.float() - full[:, lo:hi].float().cpu()).abs().max().item() <= 2e-2
            torch.testing.assert_close(l, lse[:, :, lo:hi].cpu(), atol=1e-3, rtol=1e-6)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
@pytest.mark.parametrize("exchange,make,output", [("nccl", "zigzag", "sharded"), ("nccl", "contiguous", "replicated"),
                                                  ("fused", None, "sharded"), ("fused", None, "replicated")])
def test_kv_split_four_gpus(tmp_path, exchange, make, output):
    """Four ranks: every rank's rows against the whole call (O and lse)."""
    S, H, D, world = 8192, 4, 128, 4
    path = str(tmp_path / "split4")
    port = 29800 + (os.getpid() * 7 + len(exchange) + len(output)) % 1000
    if exchange == "fused":
        mp.spawn(_fused_rank, args=(world, port, S, H, D, path, output), nprocs=world, join=True)
    else:
        mp.spawn(_nccl_rank, args=(world, port, S, H, D, path, make, output), nprocs=world, join=True)
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    full = torch.empty_like(q)
    lse = torch.empty(1, H, S, device="cuda")
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=oracle.alibi_slopes(H).cuda(),
                                        lse=lse)
    torch.cuda.synchronize()
    for r in range(world):
        res = torch.load(f"{path}.{r}")
        runs = res if exchange == "fused" else [(res["out"], res["lse"], res["rows"])]
        for out, l, (lo, hi) in runs:
            assert (out.float() - full[:, lo:hi].float().cpu()).abs().max().item() <= 2e-2
            torch.testing.assert_close(l, lse[:, :, lo:hi].cpu(), atol=1e-3, rtol=1e-6)
