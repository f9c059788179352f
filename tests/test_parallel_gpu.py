"""Key shards and the KV-split long-context path on the GPU.

* every kernel family with kv_offset / kv_total (a shard of a sequence's keys
  at its global positions) against the oracle evaluated on the same keys;
* kv_split_attention run on one GPU over all zig-zag chunks of a virtual
  4-rank split, against the unsplit kernel and the oracle;
* with two or more GPUs, the real 2-rank NCCL split against one GPU's
  unsplit result.
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


def test_kv_split_on_one_gpu_matches_unsplit():
    S, H, D = 4096, 4, 128
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    full = torch.empty_like(q)
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=slopes)
    chunks = [c for r in range(4) for c in parallel.zigzag_chunks(S, 4, r)]
    out, lse = parallel.kv_split_attention(q, [k[:, a:b] for a, b in chunks], [v[:, a:b] for a, b in chunks],
                                           [a for a, _ in chunks], S, D ** -0.5, alibi_slopes=slopes)
    torch.cuda.synchronize()
    assert (out.float() - full.float()).abs().max().item() <= 2e-2
    rows = slice(S - 256, S)
    ref = oracle.attention_ref(q[0, rows].float().cpu(), k[0].float().cpu(), v[0].float().cpu(),
                               alibi=slopes.cpu(), causal=True)
    assert_close(out[0, rows], ref, torch.bfloat16, "kv split rows")


def _nccl_rank(rank, world, port, S, H, D, path, split):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    slopes = oracle.alibi_slopes(H).cuda()
    # zig-zag: two partials per rank, merged by all-reduce; ranges: one
    # partial per rank, merged after an all-gather.
    chunks = parallel.zigzag_chunks(S, world, rank) if split == "zigzag" else parallel.kv_split_ranges(S, world, rank)
    out, lse = parallel.kv_split_attention(q, [k[:, a:b] for a, b in chunks], [v[:, a:b] for a, b in chunks],
                                           [a for a, _ in chunks], S, D ** -0.5, alibi_slopes=slopes)
    torch.cuda.synchronize()
    if rank == 0:
        torch.save({"out": out.cpu(), "lse": lse.cpu()}, path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("split", ["zigzag", "ranges"])
def test_kv_split_two_gpus_nccl(tmp_path, split):
    S, H, D = 8192, 4, 128
    path = str(tmp_path / "split.pt")
    port = 29600 + os.getpid() % 1000 + (7 if split == "ranges" else 0)
    mp.spawn(_nccl_rank, args=(2, port, S, H, D, path, split), nprocs=2, join=True)
    res = torch.load(path)
    q, k, v = (rand(1, S, H, D, seed=s).cuda() for s in range(3))
    full = torch.empty_like(q)
    lse = torch.empty(1, H, S, device="cuda")
    llmx_b200.single_mha_attention_half(full, q, k, v, D ** -0.5, alibi_slopes=oracle.alibi_slopes(H).cuda(),
                                        lse=lse)
    torch.cuda.synchronize()
    assert (res["out"].float() - full.float().cpu()).abs().max().item() <= 2e-2
    torch.testing.assert_close(res["lse"], lse.cpu(), atol=1e-3, rtol=0)


# Shapes: full and partial row runs of a block (a block takes 1024 / (D / 8)
# rows, at most 128), head dims from one 16-byte unit per row to 256 units.
@pytest.mark.parametrize("n_parts,shape,dtype", [
    (1, (2, 96, 3, 64), torch.bfloat16), (2, (2, 96, 3, 64), torch.bfloat16), (3, (2, 96, 3, 64), torch.bfloat16),
    (8, (2, 96, 3, 64), torch.bfloat16), (2, (1, 300, 2, 128), torch.float16), (3, (3, 17, 5, 8), torch.bfloat16),
    (2, (1, 40, 2, 72), torch.float16), (2, (1, 9, 1, 2048), torch.bfloat16)])
def test_merge_kernels_match_torch_merge(n_parts, shape, dtype):
    B, S, H, D = shape
    g = torch.Generator().manual_seed(n_parts)
    outs = [torch.randn(B, S, H, D, generator=g).to(dtype).cuda() for _ in range(n_parts)]
    lses = [torch.randn(B, H, S, generator=g).cuda() * 3 for _ in range(n_parts)]
    lses[0][:, :, :5] = float("-inf")  # rows the first shard never saw
    if n_parts == 1:
        lses[0][0, 0, 7] = float("-inf")  # a row nobody saw
    q = torch.empty(B, S, H, D, dtype=dtype, device="cuda")
    out, lse = parallel._merge_cuda(outs, lses, q, False, None, None)
    ref, lref = parallel.merge_partials([o.cpu() for o in outs], [l.cpu() for l in lses])
    torch.cuda.synchronize()
    assert (out.float().cpu() - ref).abs().max().item() <= 2e-2
    fin = torch.isfinite(lref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    torch.testing.assert_close(lse.cpu()[fin], lref[fin], atol=1e-4, rtol=0)
