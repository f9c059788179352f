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


def measure_e2e(w, inp, steps, warmup, stream):
    """Same call through the public API with host-resident inputs and output."""
    import llmx_b200

    qh = inp.q.cpu().pin_memory()
    kh = inp.k.cpu().pin_memory()
    vh = inp.v.cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    qd, kd, vd = torch.empty_like(inp.q), torch.empty_like(inp.k), torch.empty_like(inp.v)
    od = torch.empty_like(inp.q)
    kw = dict(alibi_slopes=inp.alibi, causal=w.causal, q_lens=inp.q_lens, kv_lens=inp.kv_lens)
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
            llmx_b200.single_mha_attention_half(od, qd, kd, vd, w.sm_scale, **kw)
            oh.copy_(od, non_blocking=True)
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
    """A bounded, seeded sample of (b, h) units copied to the host."""
    import random

    rng = random.Random(seed)
    units = []
    valid_b = [b for b in range(w.batch) if inp.q_lens_list[b] > 0 and inp.kv_lens_list[b] > 0]
    for _ in range(n_units):
        units.append((rng.choice(valid_b), rng.randrange(w.n_heads)))
    group = w.n_heads // w.n_kv_heads
    data = []
    for b, h in units:
        ql, kl = inp.q_lens_list[b], inp.kv_lens_list[b]
        kvh = h // group
        a = None if inp.alibi is None else inp.alibi[h : h + 1].cpu()
        data.append((inp.q[b, :ql, h : h + 1].cpu(), inp.k[b, :kl, kvh : kvh + 1].cpu(),
                     inp.v[b, :kl, kvh : kvh + 1].cpu(), a, ql, kl))
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
        res["e2e"] = {"value": work * world * n / (float(t.item()) * 1e-3) / scale, "unit": unit,
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    return res, w, inp


def bench_kv_split(steps, warmup, rank, world, device, stream, peaks):
    """Long-context prefill with its keys split over all ranks
    (parallel.kv_split_ranges, NCCL log-sum-exp merge); strong scaling: the
    job is one fixed sequence."""
    import torch.distributed as dist

    from llmx_b200 import parallel
    from llmx_b200.workloads import WORKLOADS, flops, make_inputs

    w = WORKLOADS["long_prefill_bf16_b1_h32_s32768_d128"]
    inp = make_inputs(w, device)
    S = w.q_len
    chunks = parallel.kv_split_ranges(S, world, rank)
    kc = [inp.k[:, a:b] for a, b in chunks]
    vc = [inp.v[:, a:b] for a, b in chunks]
    offs = [a for a, _ in chunks]
    times = []
    with torch.cuda.stream(stream):
        for i in range(warmup + steps):
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            parallel.kv_split_attention(inp.q, kc, vc, offs, S, w.sm_scale, alibi_slopes=inp.alibi)
            e1.record(stream)
            if i >= warmup:
                times.append((e0, e1))
    stream.synchronize()
    ms = torch.tensor([sum(a.elapsed_time(b) for a, b in times)], dtype=torch.float64, device=device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    per = float(ms.item()) / steps
    fl = flops(w, [S], [S])
    return {"kernel": "tcgen05 + NCCL lse merge", "value": fl / (per * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": per, "scaling": "strong", "chunks_per_rank": len(chunks),
            "roofline": {"bound": "tensor", "achieved": fl / world / (per * 1e-3) / 1e12,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s per GPU",
                         "frac": fl / world / (per * 1e-3) / 1e12 / peaks["bf16_tflops"]}}


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
    with ClockSampler(local) as clocks:
        head, w, inp = bench_workload(headline, args.steps, args.warmup, rank, world, device, stream, peaks, True)
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
    if world > 1 and not args.no_extra:
        extras["long_prefill_kv_split_" + str(world) + "gpu"] = bench_kv_split(
            3, min(args.warmup, 3), rank, world, device, stream, peaks)
    cpu = None
    if rank == 0 and world == 1:
        sample = cpu_units_sample(w, inp, args.cpu_units)
        rate, secs, threads = cpu_oracle_rate(w, sample, repeats=args.cpu_repeats)
        cpu = {"value": rate / (1e9 if w.is_decode else 1e12), "unit": head["unit"], "cores": threads,
               "kind": "port", "sample": f"{len(sample)} seeded (batch, head) units of {w.name}, x{args.cpu_repeats}, "
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
        "config": {"workload": w.name, "batch_per_gpu": w.batch, "heads": w.n_heads, "kv_heads": w.n_kv_heads,
                   "seq_len": w.q_len, "head_dim": w.head_dim, "causal": w.causal, "alibi": w.alibi,
                   "parallelism": f"batch x head shards over {world} GPU(s), no data-path collective",
                   "l2": "flushed between steps (256 MiB write)"},
        "kernel": head["kernel"],
        "roofline": head["roofline"],
        "e2e": head["e2e"],
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
        "config": {"workload": w.name, "batch_per_gpu": w.batch, "heads": w.n_heads, "seq_len": w.q_len,
                   "head_dim": w.head_dim, "causal": w.causal, "alibi": w.alibi},
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
