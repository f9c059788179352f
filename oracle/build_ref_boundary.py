"""Compiles the reference's own boundary sources, unchanged, against this
repository's headers and library: the drop-in check of the boundary.

TEST INFRASTRUCTURE ONLY.  Reads two files of the reference where they lie
(never copied into this repository) and writes only under oracle/_ref/:

* ``csrc/llmx_bind.cpp`` (the reference's torch binding,
  llmx_bind.cpp:1-78) -> ``oracle/_ref/llmx_ref_bind<ext>``, a torch extension
  module that calls ``llmx::llmx_single_mha_attention`` of
  ``libllmx_attn.so`` through ``include/llmx/cuda/attention/attention_api.h``;
* ``test/cuda/mha_attention_test.cpp`` (the reference's C++ smoke test,
  mha_attention_test.cpp:1-35) -> ``oracle/_ref/mha_attention_test``.

Both compile with nothing but include paths pointed at ``include/`` (no
edits, no reference headers).  The built files travel with the repository
to a GPU machine, where ``tests/test_ref_sources_gpu.py`` runs them.

    python -m oracle.build_ref_boundary [reference-root]

The reference root defaults to LLMX_REFERENCE_ROOT, else /root/reference.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
INCLUDE = os.path.join(ROOT, "include")
BIND_SRC = os.path.join("csrc", "llmx_bind.cpp")
TEST_SRC = os.path.join("test", "cuda", "mha_attention_test.cpp")


def reference_root(arg: str = None):
    root = arg or os.environ.get("LLMX_REFERENCE_ROOT") or "/root/reference"
    return root if os.path.exists(os.path.join(root, BIND_SRC)) else None


def ref_binding_path() -> str:
    import sysconfig

    return os.path.join(OUT, "llmx_ref_bind" + sysconfig.get_config_var("EXT_SUFFIX"))


def ref_test_path() -> str:
    return os.path.join(OUT, "mha_attention_test")


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd[:3])} ... failed:\n{r.stdout}\n{r.stderr}")


def build(ref_root: str = None, syntax_only: bool = False) -> dict:
    """Builds both reference sources (or, with syntax_only, only compiles
    them) against include/ and libllmx_attn.so; returns {name: path}."""
    sys.path.insert(0, ROOT)
    from llmx_b200 import build as b

    root = reference_root(ref_root)
    if root is None:
        raise FileNotFoundError("reference sources not found (pass the root or set LLMX_REFERENCE_ROOT)")
    lib = b.build()
    os.makedirs(OUT, exist_ok=True)
    out = {}
    # the reference's torch binding, module name llmx_ref_bind
    cflags, ldflags = b.torch_extension_flags("llmx_ref_bind")
    gxx = shutil.which("g++") or "g++"
    src = os.path.join(root, BIND_SRC)
    if syntax_only:
        _run([gxx, *[f for f in cflags if f != "-shared"], "-I" + INCLUDE, "-fsyntax-only", src])
    else:
        dst = ref_binding_path()
        _run([gxx, *cflags, "-I" + INCLUDE, src, "-o", dst, *ldflags, "-L" + os.path.dirname(lib), "-lllmx_attn",
              "-Wl,-rpath,$ORIGIN/../../llmx_b200"])
        out["binding"] = dst
    # the reference's C++ smoke test
    src = os.path.join(root, TEST_SRC)
    if syntax_only:
        _run([b.nvcc(), "-std=c++17", "-x", "cu", "-I" + INCLUDE, "-c", src, "-o", os.path.join(OUT, "mha.o")])
        os.remove(os.path.join(OUT, "mha.o"))
    else:
        dst = ref_test_path()
        _run([b.nvcc(), "-std=c++17", "-O2", "-x", "cu", "-I" + INCLUDE, src, "-o", dst,
              "-L" + os.path.dirname(lib), "-lllmx_attn", "-Xlinker", "-rpath=$ORIGIN/../../llmx_b200"])
        out["test"] = dst
    return out


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
