"""Benchmark of the llmx attention engine on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--no-extra]

One "step" is one attention forward over one batch of the workload.  The
headline workload is the Llama-7B-shaped causal prefill (B8 H32 S2048 D128
bf16); the padded-prefill, decode and long-context workloads are measured in
the same run and reported under "workloads".  With N > 1 (torchrun, one rank
per GPU) every rank runs its own batch of the workload with a rank-specific
seed -- the batch x head units are independent, so there is no collective on
the data path -- and `value` is the total work of all ranks over the slowest
rank's time ("scaling": "weak").

Timing: W untimed warm-up steps, then K timed steps; between steps a 256 MiB
buffer is rewritten to flush the 126 MB L2; each step's attention call is
bracketed by CUDA events on the stream it runs on; the step times are
summed and the max over ranks is taken.  `e2e` times the same call through
the public torch API with the inputs copied from pinned host memory and the
output copied back inside the timed region.  `--impl reference` times the
CPU restatement of the reference's oracle path (the reference has no CPU
kernel of its own; its CPU path is ref_attention in torch) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HEADLINE = "llama7b_prefill_bf16_b8_h32_s2048_d128"
EXTRA = ["padded_prefill_fp16_b4_h16_s1024_d64", "bloom_decode_bf16_b64_h32_kv4096_d128",
         "long_prefill_bf16_b1_h32_s32768_d128", "cpu_fp32_b1_h8_s128_d64", "gemma_prefill_bf16_b2_h16_s4096_d256"]
L2_FLUSH_BYTES = 256 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return {k: float(d[k]) for k in FALLBACK_PEAKS if k in d}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def dist_info():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _algo_and_launches(w, inp):
    import ctypes

    import llmx_b200
    from llmx_b200 import _lib, ops

    out = torch.empty_like(inp.q)
    algo = llmx_b200.selected_algo(out, inp.q, inp.k, inp.v, w.sm_scale, alibi_slopes=inp.alibi,
                                   causal=w.causal, q_lens=inp.q_lens, kv_lens=inp.kv_lens)
    p, _ = ops.build_params(out, inp.q, inp.k, inp.v, w.sm_scale, alibi_slopes=inp.alibi, causal=w.causal,
                            q_lens=inp.q_lens, kv_lens=inp.kv_lens)
    ws = ctypes.c_size_t(0)
    _lib.check(_lib.load().llmx_attn_workspace_size(ctypes.byref(p), ctypes.byref(ws)))
    launches = 2 if (algo == "decode" and ws.value > 0) else 1
    return algo, launches


def measure_device(w, inp, steps, warmup, stream):
    """Per-step CUDA-event time of the attention call, L2 flushed between steps."""
    import llmx_b200

    out = torch.empty_like(inp.q)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=inp.q.device)
    kw = dict(alibi_slopes=inp.alibi, causal=w.causal, q_lens=inp.q_lens, kv_lens=inp.kv_lens)
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            llmx_b200.single_mha_attention_half(out, inp.q, inp.k, inp.v, w.sm_scale, **kw)
            e1.record(stream)
            if i >= warmup:
                times.append((e0, e1))
    stream.synchronize()
    ms = [a.elapsed_time(b) for a, b in times]
    return ms, out


def measure_e2e(w, inp, steps, warmup, stream, chunks=8):
    """Same workload through the public host-memory API
    (llmx_b200.HostAttention: pinned host inputs and output, the batch cut
    into `chunks` whose uploads, kernels and downloads overlap on three
    streams).  Every step copies all of q, k, v up and all of o down."""
    import llmx_b200

    qh = inp.q.cpu().pin_memory()
    kh = inp.k.cpu().pin_memory()
    vh = inp.v.cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    run = llmx_b200.HostAttention(qh, kh, inp.q.device, chunks=min(chunks, w.batch))
    kw = dict(alibi_slopes=inp.alibi, causal=w.causal, q_lens=inp.q_lens, kv_lens=inp.kv_lens)
    times = []
    for i in range(warmup + steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run(oh, qh, kh, vh, w.sm_scale, stream=stream, **kw)
        e1.record(stream)
        if i >= warmup:
            times.append((e0, e1))
    stream.synchronize()
    ms = [a.elapsed_time(b) for a, b in times]
    h2d = sum(t.numel() * t.element_size() for t in (qh, kh, vh))
    d2h = oh.numel() * oh.element_size()
    return ms, h2d, d2h


def work_of(w, inp):
    from llmx_b200.workloads import decode_bytes, flops

    if w.is_decode:
        return decode_bytes(w, inp.kv_lens_list), "GB/s", 1e9
    return flops(w, inp.q_lens_list, inp.kv_lens_list), "TFLOP/s", 1e12


def cpu_units_sample(w, inp, n_units, seed=0):
    """A bounded, seeded sample of the workload copied to the host: (batch,
    head) units, or for long sequences (> 4096 rows) blocks of 512 query
    rows of a (batch, head) against the keys they see, so one sample element
    stays well under a second of CPU work."""
    import random

    rng = random.Random(seed)
    valid_b = [b for b in range(w.batch) if inp.q_lens_list[b] > 0 and inp.kv_lens_list[b] > 0]
    group = w.n_heads // w.n_kv_heads
    data = []
    for _ in range(n_units):
        b, h = rng.choice(valid_b), rng.randrange(w.n_heads)
        ql, kl = inp.q_lens_list[b], inp.kv_lens_list[b]
        r0, r1 = 0, ql
        if ql > 4096:
            r0 = rng.randrange(0, ql - 512 + 1)
            r1 = r0 + 512
        k_end = min(kl, r1 + (kl - ql)) if w.causal else kl  # keys the rows can see (bottom-right)
        kvh = h // group
        a = None if inp.alibi is None else inp.alibi[h : h + 1].cpu()
        data.append((inp.q[b, r0:r1, h : h + 1].cpu(), inp.k[b, :k_end, kvh : kvh + 1].cpu(),
                     inp.v[b, :k_end, kvh : kvh + 1].cpu(), a, r1 - r0, k_end))
    return data


def cpu_oracle_rate(w, sample, repeats=1):
    """Times the CPU oracle (the reference's ref_attention path restated) on
    `sample`; returns (work units per second, seconds, threads)."""
    import oracle
    from llmx_b200.workloads import visible_pairs

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    es = torch.tensor([], dtype=w.dtype).element_size()
    work = 0
    t0 = time.perf_counter()
    for _ in range(repeats):
        for q, k, v, a, ql, kl in sample:
            oracle.attention_ref(q, k, v, sm_scale=w.sm_scale, alibi=a, causal=w.causal)
            if w.is_decode:
                work += kl * w.head_dim * 2 * es + 2 * w.head_dim * es
            else:
                work += 4 * w.head_dim * visible_pairs(ql, kl, w.causal)
    dt = time.perf_counter() - t0
    return work / dt, dt, threads


def load_traffic(workload: str):
    """DRAM bytes per launch of the workload's kernel from a committed ncu summary
    (profiles/traffic.json, written from `ncu --metrics dram__bytes_*`), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    return json.load(open(path)).get(workload)


def bench_workload(name, steps, warmup, rank, world, device, stream, peaks, with_e2e):
    from llmx_b200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS[name]
    inp = make_inputs(w, device, seed=w.seed + 1000 * rank)
    algo, launches = _algo_and_launches(w, inp)
    work, unit, scale = work_of(w, inp)
    ms, _ = measure_device(w, inp, steps, warmup, stream)
    t_local = torch.tensor([sum(ms)], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    total_ms = float(t_local.item())
    ms_per_step = total_ms / steps
    value = work * world * steps / (total_ms * 1e-3) / scale
    per_launch = work / (statistics.mean(ms) * 1e-3) / scale  # this rank's kernel rate
    bound = "hbm" if w.is_decode else "tensor"
    peak = peaks["hbm_gbs"] if w.is_decode else peaks["bf16_tflops"]
    res = {
        "workload": name, "kernel": algo, "value": value, "unit": unit, "ms_per_step": ms_per_step,
        "launches_per_step": launches,
        "roofline": {"bound": bound, "achieved": per_launch, "peak": peak,
                     "unit": "GB/s" if w.is_decode else "TFLOP/s", "frac": per_launch / peak,
                     "traffic": load_traffic(name),
                     "algorithmic": work},
    }
    if with_e2e:
        ems, h2d, d2h = measure_e2e(w, inp, max(3, steps // 2), max(1, warmup // 2), stream)
        t = torch.tensor([sum(ems)], dtype=torch.float64, device=device)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n = len(ems)
        e2e_ms = float(t.item()) / n
        res["e2e"] = {"value": work * world * n / (float(t.item()) * 1e-3) / scale, "unit": unit,
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                      "copy_gbs": (h2d + d2h) / (e2e_ms * 1e-3) / 1e9,
                      "pipeline": "HostAttention: batch in 8 chunks, upload / kernel / download on 3 streams"}
    return res, w, inp


def _max_over_ranks(values, world, device):
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def check_parity(out, lse, q, k, v, w, alibi, rows, heads, unsplit, world, device, cpu_blocks=2, seed=0):
    """The checker of a multi-GPU leg, outside its timed region: this rank's
    output rows `rows` of heads `heads` against (1) the single-GPU unsplit
    kernel result `unsplit` on the same rows, (2) the fp32 oracle evaluated on
    this GPU over every row and head this rank holds (oracle.attention_ref_chunked),
    (3) the CPU oracle on `cpu_blocks` seeded 128-row blocks.  Tolerances: bf16
    <= 2e-2 max-abs and <= 1e-2 mean-relative (the oracle), lse <= 2e-3.
    Returns the parity block, worst case over ranks."""
    import random

    import oracle

    r0, r1 = rows
    hs = list(heads)
    ref, lref = oracle.attention_ref_chunked(q, k, v, alibi=alibi, causal=w.causal, rows=(r0, r1), heads=hs)
    err = (out.float() - ref).abs()
    max_abs = float(err.max()) if err.numel() else 0.0
    mean_rel = float(err.mean() / ref.abs().mean().clamp_min(1e-12)) if err.numel() else 0.0
    fin = torch.isfinite(lref)
    # lse reaches ~3e4 with ALiBi (one fp32 ulp ~2e-3): error beyond 1e-6 relative
    lse_err = float(((lse[fin] - lref[fin]).abs() - 1e-6 * lref[fin].abs()).clamp_min(0).max()) if fin.any() else 0.0
    vs_unsplit = float((out.float() - unsplit.float()).abs().max()) if out.numel() else 0.0
    rng = random.Random(seed + r0)
    cpu_err = 0.0
    for _ in range(cpu_blocks if r1 > r0 else 0):
        h = rng.choice(hs)
        a = rng.randrange(r0, r1)
        a = min(a, max(r0, r1 - 128))
        e = min(r1, a + 128)
        kv_end = e + (w.kv_len - w.q_len) if w.causal else w.kv_len
        ro = oracle.attention_ref(q[0, a:e, h:h + 1].float().cpu(), k[0, :kv_end, h:h + 1].float().cpu(),
                                  v[0, :kv_end, h:h + 1].float().cpu(), sm_scale=w.sm_scale,
                                  alibi=None if alibi is None else alibi[h:h + 1].cpu(), causal=w.causal)
        got = out[0, a - r0:e - r0, hs.index(h):hs.index(h) + 1].float().cpu()
        cpu_err = max(cpu_err, float((got - ro).abs().max()))
    worst = _max_over_ranks([max_abs, mean_rel, lse_err, vs_unsplit, cpu_err], world, device)
    ok = worst[0] <= 2e-2 and worst[1] <= 1e-2 and worst[2] <= 2e-3 and worst[4] <= 2e-2
    return {"max_abs": worst[0], "mean_rel": worst[1], "lse_max_abs_beyond_1e-6_rel": worst[2], "vs_unsplit_max_abs": worst[3],
            "cpu_oracle_blocks_max_abs": worst[4], "cpu_oracle_blocks_per_rank": cpu_blocks, "ok": bool(ok),
            "checked": "every row and head each rank holds vs the fp32 oracle on the GPU; the single-GPU kernel; "
                       "seeded 128-row blocks vs the CPU oracle"}


def _timed(fn, steps, warmup, stream, world, sync=None):
    """Per-step CUDA-event time of fn() on `stream` (a barrier before each
    step when world > 1); returns (ms per step, max over ranks; per-step
    phase marks from the last step)."""
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            if world > 1:
                import torch.distributed as dist

                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            marks = fn()
            e1.record(stream)
            if i >= warmup:
                times.append((e0, e1, marks))
    stream.synchronize()
    total = sum(a.elapsed_time(b) for a, b, _ in times)
    phases = {}
    for e0, _, marks in times:
        prev = e0
        for name, ev in marks or []:
            phases[name] = phases.get(name, 0.0) + prev.elapsed_time(ev) / len(times)
            prev = ev
    names = sorted(phases)
    vals = _max_over_ranks([total / steps] + [phases[n] for n in names], world, stream.device)
    return vals[0], dict(zip(names, vals[1:]))


def bench_kv_split(steps, warmup, rank, world, device, stream, peaks, unsplit):
    """Long-context prefill (B1 H32 S32768 D128 bf16, causal + ALiBi) with its
    keys split over all ranks (parallel.KVSplitPlan.contiguous: one
    work-balanced key range per rank, each rank computing only the rows that
    can see its keys, merged per row slice by the library's log-sum-exp
    kernel); strong scaling.  Two exchanges are timed: "fused" (the attention
    kernel writes each row straight into the owning rank's buffer over NVLink
    through CUDA IPC, then one barrier) -- the leg's headline -- and "nccl"
    (row slices sent point to point by NCCL after the kernel); each with the
    output row-sharded and replicated (plus an NCCL all-gather)."""
    from llmx_b200 import parallel
    from llmx_b200.workloads import WORKLOADS, flops, make_inputs

    w = WORKLOADS["long_prefill_bf16_b1_h32_s32768_d128"]
    inp = make_inputs(w, device)
    S = w.q_len
    plan = parallel.KVSplitPlan.contiguous(S, world)
    mine = plan.chunks[rank]
    kc = [inp.k[:, a:b] for a, b in mine]
    vc = [inp.v[:, a:b] for a, b in mine]
    fl = flops(w, [S], [S])
    ex = parallel.PeerExchange(plan, 1, w.n_heads, w.head_dim, w.dtype, device)
    res = {"kernel": "tcgen05 (row-restricted partial) + row-slice exchange + lse merge kernel",
           "plan": {"key_ranges": [list(c) for c in plan.chunks], "first_rows": [plan.first_row(r) for r in range(world)],
                    "slice_rows": plan.slice_rows}}
    for name, exch in (("fused", ex), ("nccl", None)):
        for output in ("sharded", "replicated"):
            holder = {}

            def step():
                marks = []
                holder["r"] = parallel.kv_split_attention(inp.q, kc, vc, plan, w.sm_scale, alibi_slopes=inp.alibi,
                                                          output=output, timings=marks, exchange=exch)
                return marks

            per, phases = _timed(step, steps, warmup, stream, world)
            key = f"{name}_{output}"
            res[key] = {"value": fl / (per * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": per,
                        "phase_ms_max_over_ranks": phases}
            if output == "sharded":
                out, lse, (lo, hi) = holder["r"]
                res[key]["parity"] = check_parity(out, lse, inp.q, inp.k, inp.v, w, inp.alibi, (lo, hi),
                                                  range(w.n_heads), unsplit[:, lo:hi], world, device)
            del holder
    ex.close()
    head = res["fused_sharded"]
    res.update({"value": head["value"], "unit": "TFLOP/s", "ms_per_step": head["ms_per_step"], "scaling": "strong",
                "parity": head["parity"],
                "output": "row-sharded (each rank holds the merged rows of its slice), fused exchange; the other "
                          "three lines: replicated output (all-gather) and NCCL point-to-point exchange",
                "roofline": {"bound": "tensor", "achieved": fl / world / (head["ms_per_step"] * 1e-3) / 1e12,
                             "peak": peaks["bf16_tflops"], "unit": "TFLOP/s per GPU",
                             "frac": fl / world / (head["ms_per_step"] * 1e-3) / 1e12 / peaks["bf16_tflops"]}})
    return res


def bench_head_split(steps, warmup, rank, world, device, stream, peaks, unsplit):
    """Long-context prefill with its 32 heads dealt over the ranks
    (parallel.head_range: 4 heads per GPU at 8 GPUs), no collective; strong
    scaling of one fixed sequence."""
    import llmx_b200
    from llmx_b200 import parallel
    from llmx_b200.workloads import WORKLOADS, flops, make_inputs

    w = WORKLOADS["long_prefill_bf16_b1_h32_s32768_d128"]
    inp = make_inputs(w, device)
    S = w.q_len
    h0, h1 = parallel.head_range(w.n_heads, world, rank)
    out = torch.empty_like(inp.q[:, :, h0:h1])

    def step():
        llmx_b200.single_mha_attention_half(out, inp.q[:, :, h0:h1], inp.k[:, :, h0:h1], inp.v[:, :, h0:h1],
                                            w.sm_scale, alibi_slopes=inp.alibi[h0:h1])
        return None

    per, _ = _timed(step, steps, warmup, stream, world)
    fl = flops(w, [S], [S])
    lse = torch.empty(1, h1 - h0, S, device=device)
    llmx_b200.single_mha_attention_half(out, inp.q[:, :, h0:h1], inp.k[:, :, h0:h1], inp.v[:, :, h0:h1],
                                        w.sm_scale, alibi_slopes=inp.alibi[h0:h1], lse=lse)
    parity = check_parity(out, lse, inp.q, inp.k, inp.v, w, inp.alibi, (0, S), range(h0, h1), unsplit[:, :, h0:h1],
                          world, device)
    return {"kernel": "tcgen05, heads [h0, h1) per rank, no collective", "heads_per_rank": h1 - h0,
            "value": fl / (per * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": per, "scaling": "strong",
            "roofline": {"bound": "tensor", "achieved": fl / world / (per * 1e-3) / 1e12,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s per GPU",
                         "frac": fl / world / (per * 1e-3) / 1e12 / peaks["bf16_tflops"]},
            "parity": parity}


def bench_strong_units(steps, warmup, rank, world, device, stream, peaks, name=None):
    """One fixed job (the same seed on every rank) whose (batch, head) units
    are dealt over the ranks, no collective; strong scaling.  Units are split
    by work (parallel.shard_units_weighted): for a prefill each sequence's
    heads weigh its visible (query, key) pairs, for a decode its key length,
    so padded batches with unequal lengths still balance; in granules of whole
    sequences or head blocks (parallel.launch_granule), so that a rank runs
    one launch per run of sequences.  L2 flushed between
    steps.  Parity: each rank's units against the whole job on one GPU --
    bit-identical for a prefill (a unit's result does not depend on the other
    units); for a decode the split-KV plan depends on how many units a launch
    holds, so the check is the tolerance of the parity tests."""
    import llmx_b200
    from llmx_b200 import parallel
    from llmx_b200.workloads import WORKLOADS, make_inputs, visible_pairs

    w = WORKLOADS[name or HEADLINE]
    inp = make_inputs(w, device)  # same seed on every rank: one job
    if w.is_decode:
        weights = list(inp.kv_lens_list)
    else:
        weights = [visible_pairs(ql, kl, w.causal) for ql, kl in zip(inp.q_lens_list, inp.kv_lens_list)]
    group = w.n_heads // w.n_kv_heads
    granule = parallel.launch_granule(w.batch, w.n_heads, world, group)
    start, end = parallel.shard_units_weighted(weights, w.n_heads, world, rank, align=granule)
    kw = dict(alibi_slopes=inp.alibi, causal=w.causal, q_lens=inp.q_lens, kv_lens=inp.kv_lens)
    out = torch.zeros_like(inp.q)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    n_launch = [0]
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            if world > 1:
                import torch.distributed as dist

                dist.barrier()
            flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            n_launch[0] = parallel.run_units(out, inp.q, inp.k, inp.v, start, end, w.sm_scale, **kw)
            e1.record(stream)
            if i >= warmup:
                times.append((e0, e1))
    stream.synchronize()
    per = _max_over_ranks([sum(a.elapsed_time(b) for a, b in times) / steps], world, device)[0]
    work, unit, scale = work_of(w, inp)
    full = torch.empty_like(inp.q)
    llmx_b200.single_mha_attention_half(full, inp.q, inp.k, inp.v, w.sm_scale, **kw)
    torch.cuda.synchronize(device)
    runs = parallel.unit_runs(start, end, w.n_heads)
    same = all(torch.equal(out[b0:b1, :, h0:h1], full[b0:b1, :, h0:h1]) for b0, b1, h0, h1 in runs)
    max_abs = max([(out[b0:b1, :, h0:h1].float() - full[b0:b1, :, h0:h1].float()).abs().max().item()
                   for b0, b1, h0, h1 in runs] or [0.0])
    same_all, max_abs_all = _max_over_ranks([0.0 if same else 1.0, max_abs], world, device)
    ok = same_all == 0.0 if not w.is_decode else max_abs_all <= 2e-2
    bound = "hbm" if w.is_decode else "tensor"
    peak = peaks["hbm_gbs"] if w.is_decode else peaks["bf16_tflops"]
    per_gpu = work / world / (per * 1e-3) / scale
    return {"kernel": f"{'split-KV decode' if w.is_decode else 'tcgen05'} on this rank's (batch, head) units",
            "workload": w.name, "units_per_rank": end - start, "unit_granule": granule,
            "launches_per_step": n_launch[0],
            "value": work / (per * 1e-3) / scale, "unit": unit, "ms_per_step": per, "scaling": "strong",
            "roofline": {"bound": bound, "achieved": per_gpu, "peak": peak, "unit": f"{unit} per GPU",
                         "frac": per_gpu / peak},
            "parity": {"bitwise_equal_to_single_gpu_call": same_all == 0.0, "max_abs_vs_single_gpu_call": max_abs_all,
                       "ok": ok}}


def bench_convert(steps, warmup, rank, world, device, stream, peaks):
    """The dtype-convert op (to_bf16 of an fp32 tensor, 256 Mi elements = 1 GiB
    in, 512 MiB out; both larger than L2): HBM-bound, bytes read + written."""
    import llmx_b200

    n = 256 << 20
    g = torch.Generator(device=device).manual_seed(7 + rank)
    x = torch.randn(n, generator=g, device=device)
    out = torch.empty(n, dtype=torch.bfloat16, device=device)
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            llmx_b200.convert(x, torch.bfloat16, out=out)
            e1.record(stream)
            if i >= warmup:
                times.append((e0, e1))
    stream.synchronize()
    ms = [a.elapsed_time(b) for a, b in times]
    t = torch.tensor([sum(ms)], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    nbytes = n * (4 + 2)
    per = float(t.item()) / steps
    achieved = nbytes / (statistics.mean(ms) * 1e-3) / 1e9
    del x, out
    return {"kernel": "convert", "value": nbytes * world / (per * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": per,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": None, "algorithmic": nbytes}}


def headline_config(w, world):
    """The `config` of the headline line, shared by both arms."""
    return {"workload": w.name, "batch_per_gpu": w.batch, "heads": w.n_heads, "kv_heads": w.n_kv_heads,
            "seq_len": w.q_len, "head_dim": w.head_dim, "causal": w.causal, "alibi": w.alibi,
            "parallelism": f"replica per GPU: each of {world} GPU(s) runs the whole workload on its own seed, "
                           "no collective (weak scaling); the fixed job split over the GPUs is under "
                           f"workloads.llama7b_prefill_strong_{world}gpu",
            "l2": "flushed between steps (256 MiB write)"}


def run_ours(args):
    rank, world, local = dist_info()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    import llmx_b200  # noqa: F401  (loads libllmx_attn.so; fails loudly if missing)

    peaks, peak_src = load_peaks()
    stream = torch.cuda.Stream(device)
    headline = args.workload or HEADLINE
    if args.profile_only:
        args.no_extra = True
    with ClockSampler(local) as clocks:
        head, w, inp = bench_workload(headline, args.steps, args.warmup, rank, world, device, stream, peaks,
                                      not args.profile_only)
    extras = {}
    if not args.no_extra:
        for name in EXTRA:
            if name == headline:
                continue
            steps = 3 if name.startswith("long_") else args.steps
            r, _, _ = bench_workload(name, steps, min(args.warmup, 3) if name.startswith("long_") else args.warmup,
                                     rank, world, device, stream, peaks, False)
            extras[name] = {k: r[k] for k in ("kernel", "value", "unit", "ms_per_step", "roofline")}
    if not args.no_extra:
        extras["dtype_convert_fp32_to_bf16_256Mi"] = bench_convert(args.steps, args.warmup, rank, world, device,
                                                                   stream, peaks)
    if not args.no_extra:
        extras[f"llama7b_prefill_strong_{world}gpu"] = bench_strong_units(args.steps, args.warmup, rank, world,
                                                                         device, stream, peaks)
        extras[f"padded_prefill_strong_{world}gpu"] = bench_strong_units(
            args.steps, args.warmup, rank, world, device, stream, peaks, "padded_prefill_fp16_b4_h16_s1024_d64")
        extras[f"bloom_decode_strong_{world}gpu"] = bench_strong_units(
            args.steps, args.warmup, rank, world, device, stream, peaks, "bloom_decode_bf16_b64_h32_kv4096_d128")
    if world > 1 and not args.no_extra:
        # the single-GPU result every rank checks its share of the long sequence against
        from llmx_b200.workloads import WORKLOADS as _W, make_inputs as _mk

        lw = _W["long_prefill_bf16_b1_h32_s32768_d128"]
        li = _mk(lw, device)
        unsplit = torch.empty_like(li.q)
        llmx_b200.single_mha_attention_half(unsplit, li.q, li.k, li.v, lw.sm_scale, alibi_slopes=li.alibi)
        torch.cuda.synchronize(device)
        del li
        extras[f"long_prefill_kv_split_{world}gpu"] = bench_kv_split(3, min(args.warmup, 3), rank, world, device,
                                                                     stream, peaks, unsplit)
        extras[f"long_prefill_head_split_{world}gpu"] = bench_head_split(3, min(args.warmup, 3), rank, world,
                                                                         device, stream, peaks, unsplit)
        del unsplit
    cpu = None
    if rank == 0 and world == 1 and not args.profile_only:
        sample = cpu_units_sample(w, inp, args.cpu_units)
        rate, secs, threads = cpu_oracle_rate(w, sample, repeats=args.cpu_repeats)
        cpu = {"value": rate / (1e9 if w.is_decode else 1e12), "unit": head["unit"], "cores": threads,
               "kind": "port", "sample": f"{len(sample)} seeded (batch, head) units (512-row blocks past 4096 rows) of {w.name}, x{args.cpu_repeats}, "
                                         f"through the CPU oracle: {secs:.1f} s on {threads} threads"}
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak_unit = head["roofline"]["unit"]
    head["roofline"]["peak_source"] = peak_src
    line = {
        "metric": "attention TFLOP/s/GPU (% BF16 tensor peak); decode HBM GB/s; 1-8 GPUs",
        "value": head["value"], "unit": head["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[w.dtype],
        "data": "synthetic: seeded N(0,1) inputs of the workload's shape (rank-specific seed per GPU)",
        "config": headline_config(w, world),
        "kernel": head["kernel"],
        "roofline": head["roofline"],
        "e2e": head.get("e2e"),
        "gpu_launches": head["launches_per_step"] * args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "workloads": extras,
    }
    assert peak_unit
    print(json.dumps(line), file=RESULT_OUT, flush=True)


def run_reference(args):
    """The reference arm: its CPU path (ref_attention, restated in oracle/) on
    the host cores, rank 0 only."""
    rank, world, _ = dist_info()
    if rank != 0:
        return
    from llmx_b200.workloads import WORKLOADS, make_inputs

    w = WORKLOADS[args.workload or HEADLINE]
    inp = make_inputs(w, "cpu") if not w.device_inputs else None
    if inp is None:
        from dataclasses import replace

        inp = make_inputs(replace(w, device_inputs=False), "cpu")
    sample = cpu_units_sample(w, inp, args.ref_units)
    rates = []
    for i in range(args.warmup + args.steps):
        rate, secs, threads = cpu_oracle_rate(w, sample)
        if i >= args.warmup:
            rates.append((rate, secs))
    scale = 1e9 if w.is_decode else 1e12
    unit = "GB/s" if w.is_decode else "TFLOP/s"
    tot_secs = sum(s for _, s in rates)
    value = sum(r * s for r, s in rates) / tot_secs / scale
    line = {
        "impl": "reference",
        "metric": "attention TFLOP/s/GPU (% BF16 tensor peak); decode HBM GB/s; 1-8 GPUs",
        "value": value, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot_secs / len(rates) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic: seeded N(0,1) inputs of the workload's shape",
        "config": headline_config(w, world),
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                         "sample": f"each step: {len(sample)} seeded (batch, head) units of {w.name} through "
                                   f"the reference oracle's CPU path (ref_attention restated, fp32 torch)"},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), file=RESULT_OUT, flush=True)


# The result line goes to the process's original standard output; everything
# else written to file descriptor 1 (NCCL's version banner, library logs,
# stray prints) is sent to standard error, so stdout carries the one JSON line.
RESULT_OUT = sys.stdout


def main():
    global RESULT_OUT
    sys.stdout.flush()
    RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=None)
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary workloads")
    ap.add_argument("--profile-only", action="store_true",
                    help="device-timed steps of the one workload only (no e2e, cpu_baseline or extras): for ncu")
    ap.add_argument("--cpu-units", type=int, default=64, help="units in the cpu_baseline sample")
    ap.add_argument("--cpu-repeats", type=int, default=6, help="passes over the cpu_baseline sample")
    ap.add_argument("--ref-units", type=int, default=32, help="units per step of the reference arm")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
