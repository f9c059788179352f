"""Loads the golden fixtures written by tests/golden/make_golden.py."""
import json
import os

import numpy as np
import torch

from cases import GoldenCase

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden():
    man = json.load(open(os.path.join(HERE, "ref_attention_golden.json")))
    arr = np.load(os.path.join(HERE, "ref_attention_golden.npz"))
    out = []
    for e in man["cases"]:
        fields = {k: e[k] for k in GoldenCase.__dataclass_fields__}
        c = GoldenCase(**fields)
        out.append((c, e, arr[c.name + "/idx"], arr[c.name + "/val"]))
    return out


def ulp_tol(dtype: str, ref: np.ndarray) -> np.ndarray:
    """One unit in the last place of the output dtype at |ref| (plus a floor)."""
    bits = {"fp32": 23, "fp16": 10, "bf16": 7}[dtype]
    mag = np.maximum(np.abs(ref), 2.0 ** -14)
    return np.exp2(np.floor(np.log2(mag)) - bits) + 1e-6


def to_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().reshape(-1).numpy()
