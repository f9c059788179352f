"""Generate the golden attention fixtures from the reference's own oracle.

Run where the reference source is available, naming its root (the
directory holding ``csrc/test_attention.py``) as the one argument or in
LLMX_REFERENCE_ROOT:

    python tests/golden/make_golden.py <reference-root>

It reads ``ref_attention`` out of ``csrc/test_attention.py`` (lines 41-93)
with ``ast`` -- importing that module would start its torch JIT build
(test_attention.py:13-38) -- and runs it on CPU torch for every case in
``cases.py``.  Paths the reference's signature cannot express directly are
composed from single-sequence calls, exactly as the reference itself would be
driven one sequence at a time:

* padded batches: one call per sequence on its first kv_len keys;
* non-causal rows: one call per query row i on q[i:i+1] and the sequence's
  kv_len keys (bottom-right alignment then makes every key visible).

Outputs are written to ``ref_attention_golden.npz`` (values) and
``ref_attention_golden.json`` (case parameters, input checksums, output sums).
The CPU-runnable fp32 workload is stored whole; every other case as 1024
seeded samples of its flattened output.
"""

from __future__ import annotations

import ast
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from cases import all_cases, make_inputs  # noqa: E402

N_SAMPLES = 1024
FULL_CASES = ("c1_fp32_b1_h8_s128_d64_alibi",)  # the CPU-runnable workload is stored whole


def load_ref_attention(ref_root: str):
    path = os.path.join(ref_root, "csrc", "test_attention.py")
    tree = ast.parse(open(path).read(), filename=path)
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "ref_attention"]
    if len(fn) != 1:
        raise RuntimeError("ref_attention not found in " + path)
    mod = ast.Module(body=fn, type_ignores=[])
    ns = {"torch": torch, "math": __import__("math")}
    exec(compile(mod, path, "exec"), ns)
    return ns["ref_attention"]


def run_case(ref_attention, c):
    q, k, v, slopes = make_inputs(c)
    kw = dict(logits_soft_cap=c.logits_soft_cap, sliding_window=c.sliding_window, alibi_slopes=slopes)
    if c.kind == "single":
        return q, k, v, ref_attention(q, k, v, **kw)
    out = torch.zeros_like(q)
    for b in range(c.batch):
        ql = c.q_lens[b] if c.q_lens else c.q_len
        kl = c.kv_lens[b] if c.kv_lens else c.kv_len
        if ql == 0 or kl == 0:
            continue
        if c.causal:
            out[b, :ql] = ref_attention(q[b, :ql], k[b, :kl], v[b, :kl], **kw)
        else:
            for i in range(ql):
                out[b, i : i + 1] = ref_attention(q[b, i : i + 1], k[b, :kl], v[b, :kl], **kw)
    return q, k, v, out


def checksum(t: torch.Tensor) -> float:
    return float(t.double().sum().item())


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLMX_REFERENCE_ROOT")
    if not ref_root:
        sys.exit("usage: make_golden.py <reference-root>  (or set LLMX_REFERENCE_ROOT)")
    torch.set_grad_enabled(False)
    ref_attention = load_ref_attention(ref_root)
    arrays, manifest = {}, []
    for c in all_cases():
        q, k, v, out = run_case(ref_attention, c)
        flat = out.float().reshape(-1)
        entry = c.to_json()
        entry["input_checksums"] = [checksum(q), checksum(k), checksum(v)]
        entry["out_shape"] = list(out.shape)
        entry["out_sum"] = float(flat.double().sum())
        entry["out_abs_sum"] = float(flat.double().abs().sum())
        if c.name in FULL_CASES or flat.numel() <= N_SAMPLES:
            idx = np.arange(flat.numel(), dtype=np.int32)
        else:
            seed = int(hashlib.sha256(c.name.encode()).hexdigest()[:8], 16)
            rng = np.random.default_rng(seed)
            idx = np.sort(rng.choice(flat.numel(), size=N_SAMPLES, replace=False)).astype(np.int32)
        arrays[c.name + "/idx"] = idx
        arrays[c.name + "/val"] = flat.numpy()[idx].astype(np.float32)
        manifest.append(entry)
        print(f"{c.name:40s} out{tuple(out.shape)} stored {idx.size}")
    np.savez_compressed(os.path.join(HERE, "ref_attention_golden.npz"), **arrays)
    with open(os.path.join(HERE, "ref_attention_golden.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                   "source": "csrc/test_attention.py:41-93 (ref_attention)", "cases": manifest}, f, indent=1)


if __name__ == "__main__":
    main()
