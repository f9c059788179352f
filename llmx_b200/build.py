"""Builds libllmx_attn.so in-tree with nvcc for sm_100a.

    python -m llmx_b200.build          # incremental
    python -m llmx_b200.build --force  # rebuild everything

Each CUDA/C++ source is compiled to an object under llmx_b200/_build/ (only
when it or a header changed) and linked into llmx_b200/libllmx_attn.so.
No JIT cache is involved: the built library sits next to the package.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libllmx_attn.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]
# Kernel and C-ABI units export only what include/llmx_attn.h marks LLMX_API;
# the C++ Tensor / attention API units export their whole public surface.
HIDDEN = ["-Xcompiler", "-fvisibility=hidden"]
SOURCES = ["attn_api.cu", "attn_simt.cu", "attn_decode.cu", "attn_sm100.cu", "attn_merge.cu", "llmx_convert.cu",
           "llmx_tensor.cu", "attention_api.cu", "llmx_ops.cu"]
# The C++ Tensor / attention / registry units; every other unit is compiled hidden.
CXX_API_UNITS = ("llmx_tensor.cu", "attention_api.cu", "llmx_ops.cu")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    hs += glob.glob(os.path.join(INCLUDE, "**", "*.h"), recursive=True)
    return hs


def _stale(obj: str, src: str, headers) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *headers])


def _compile(src: str, obj: str, extra) -> str:
    vis = [] if os.path.basename(src) in CXX_API_UNITS else HIDDEN
    cmd = [nvcc(), *NVCC_FLAGS, *vis, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    jobs = []
    objs = []
    for name in SOURCES:
        src = os.path.join(CSRC, name)
        obj = os.path.join(BUILD, name + ".o")
        objs.append(obj)
        if force or _stale(obj, src, headers):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, list(extra_flags)): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg.strip():
                    print(f"[{os.path.basename(futs[f])}]\n{msg}", file=sys.stderr)
    if jobs or force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


BIND_SRC = os.path.join(CSRC, "llmx_bind.cpp")


def binding_path() -> str:
    import sysconfig

    return os.path.join(PKG, "llmx_bind" + sysconfig.get_config_var("EXT_SUFFIX"))


def torch_extension_flags(module: str):
    """Compiler and linker flags of a torch extension module named `module`
    (what torch.utils.cpp_extension would pass, without its JIT cache)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    inc = [*ce.include_paths(), os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include"),
           sysconfig.get_paths()["include"]]
    cflags = ["-O2", "-std=c++17", "-fPIC", "-shared", f"-DTORCH_EXTENSION_NAME={module}",
              "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
              *["-I" + d for d in inc]]
    tlib = ce.library_paths()[0]
    ldflags = ["-L" + tlib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
               "-Wl,-rpath," + tlib]
    return cflags, ldflags


def build_binding(force: bool = False) -> str:
    """Builds the torch binding (csrc/llmx_bind.cpp) as the extension module
    llmx_b200.llmx_bind, linked against libllmx_attn.so next to it."""
    lib = build()
    out = binding_path()
    deps = [BIND_SRC, lib, os.path.join(INCLUDE, "llmx_attn.h")]
    if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps):
        return out
    cflags, ldflags = torch_extension_flags("llmx_bind")
    gxx = shutil.which("g++") or "g++"
    tmp = out + ".tmp"
    cmd = [gxx, *cflags, "-I" + INCLUDE, BIND_SRC, "-o", tmp, *ldflags, "-L" + PKG, "-lllmx_attn",
           "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch binding build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    args = sys.argv[1:]
    print(build(force="--force" in args, verbose="-v" in args or "--verbose" in args))
    if "--no-binding" not in args:
        print(build_binding(force="--force" in args))
