"""C-ABI checks that need no GPU: the library loads, exports every function
include/llmx_attn.h declares, the ctypes struct matches the C layout, and
host-side validation / kernel selection behave like the reference's checks
(llmx_bind.cpp:41-58, attention_api.cpp:22-25)."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from llmx_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llmx_attn.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"LLMX_API\s+[\w\s\*]+?\b(llmx_\w+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_exported_symbols_are_only_the_abi_and_cpp_api():
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    out = subprocess.run([nm, "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    c_syms = {l.split()[-1] for l in out.splitlines() if " T llmx_" in l}
    assert c_syms == set(declared_functions())


def test_struct_layout_matches_c():
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = r"""
#include <stdio.h>
#include <stddef.h>
#include "llmx_attn.h"
#define O(f) printf("%s %zu\n", #f, offsetof(llmx_attn_params, f));
int main(void) {
  printf("size %zu\n", sizeof(llmx_attn_params));
  O(dtype) O(algo) O(q) O(o) O(q_stride) O(o_stride) O(q_lens) O(alibi_slopes) O(sm_scale)
  O(causal) O(logits_soft_cap) O(lse) O(workspace) O(workspace_bytes) O(kv_offset) O(kv_total)
  return 0;
}
"""
    tmp = os.path.join(ROOT, "llmx_b200", "_build")
    os.makedirs(tmp, exist_ok=True)
    c_path, exe = os.path.join(tmp, "layout.c"), os.path.join(tmp, "layout")
    open(c_path, "w").write(src)
    subprocess.run([gcc, "-I", os.path.join(ROOT, "include"), c_path, "-o", exe], check=True)
    lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in lines if l.strip())
    assert int(got.pop("size")) == ctypes.sizeof(_lib.AttnParams)
    for f, off in got.items():
        assert getattr(_lib.AttnParams, f).offset == int(off), f


def _params(**over):
    lib = _lib.load()
    p = _lib.AttnParams()
    assert lib.llmx_attn_params_init(ctypes.byref(p)) == 0
    p.dtype, p.batch, p.n_heads, p.n_kv_heads, p.head_dim = 2, 2, 8, 2, 128
    p.max_q_len, p.max_kv_len = 256, 256
    # fake, 16-byte aligned addresses: nothing is dereferenced on the host
    p.q, p.k, p.v, p.o = 0x10000, 0x20000, 0x30000, 0x40000
    p.sm_scale = 128 ** -0.5
    assert lib.llmx_attn_set_contiguous_strides(ctypes.byref(p)) == 0
    for k, v in over.items():
        setattr(p, k, v)
    return p


def lib_ok(p):
    return _lib.load().llmx_attn_set_contiguous_strides(ctypes.byref(p)) == 0


def _select(p):
    out = ctypes.c_int32(-1)
    st = _lib.load().llmx_attn_select_algo(ctypes.byref(p), ctypes.byref(out))
    return st, out.value


def test_defaults_and_contiguous_strides():
    p = _params()
    assert p.causal == 1 and p.sliding_window == -1 and p.algo == 0
    assert list(p.q_stride) == [256 * 8 * 128, 8 * 128, 128]
    assert list(p.k_stride) == [256 * 2 * 128, 2 * 128, 128]


@pytest.mark.parametrize("field,value", [
    ("dtype", 7), ("batch", 0), ("n_heads", 0), ("n_kv_heads", 3), ("head_dim", 0),
    ("head_dim", 257), ("max_q_len", 0), ("max_kv_len", 0), ("q", 0), ("algo", 9),
    ("sm_scale", float("nan")), ("kv_offset", -1), ("kv_total", -5),
])
def test_invalid_arguments_rejected(field, value):
    lib = _lib.load()
    p = _params(**{field: value})
    st = lib.llmx_attn_fwd(ctypes.byref(p), None)
    assert st == 1, _lib.STATUS_NAMES.get(st)
    assert lib.llmx_attn_last_error()  # a message is recorded


def test_negative_stride_rejected():
    p = _params()
    p.k_stride[1] = -1
    assert _lib.load().llmx_attn_fwd(ctypes.byref(p), None) == 1


def test_algorithm_selection():
    assert _select(_params()) == (0, _lib.ALGO["tcgen05"])
    assert _select(_params(max_q_len=1)) == (0, _lib.ALGO["decode"])
    assert _select(_params(dtype=0)) == (0, _lib.ALGO["simt"])
    assert _select(_params(head_dim=80)) == (0, _lib.ALGO["simt"])
    # head_dim 256 prefill runs on the tensor-core kernel (one query tile per work item)
    p256 = _params(head_dim=256)
    assert lib_ok(p256) and _select(p256) == (0, _lib.ALGO["tcgen05"])
    # unaligned base pointer: vector/TMA paths refuse, SIMT takes it
    assert _select(_params(q=0x10002)) == (0, _lib.ALGO["simt"])
    # forcing a path that cannot run the request is an error, not a fallback
    assert _select(_params(algo=_lib.ALGO["decode"]))[0] == 2
    assert _select(_params(dtype=0, algo=_lib.ALGO["tcgen05"]))[0] == 2


def test_workspace_size_for_split_kv_decode():
    lib = _lib.load()
    p = _params(max_q_len=1, max_kv_len=4096, batch=64, n_heads=32, n_kv_heads=32)
    ws = ctypes.c_size_t(0)
    assert lib.llmx_attn_workspace_size(ctypes.byref(p), ctypes.byref(ws)) == 0
    # 16 splits of 256 keys: partial O and lse in fp32 for every (split, b, h)
    assert ws.value == 16 * 64 * 32 * (128 + 1) * 4
    # the tensor-core prefill asks for its work counter (256 bytes); SIMT for nothing
    p2 = _params()
    assert lib.llmx_attn_workspace_size(ctypes.byref(p2), ctypes.byref(ws)) == 0 and ws.value == 256
    p3 = _params(dtype=0)
    assert lib.llmx_attn_workspace_size(ctypes.byref(p3), ctypes.byref(ws)) == 0 and ws.value == 0


def test_status_strings():
    lib = _lib.load()
    for code in _lib.STATUS_NAMES:
        assert lib.llmx_status_string(code)
    assert lib.llmx_attn_abi_version() == 3


def test_scatter_and_ipc_arguments_checked_before_any_device_work():
    """The row-scatter and IPC entry points reject bad arguments on the host
    (no GPU needed), and closing or freeing NULL does nothing."""
    lib = _lib.load()
    p = _params()
    x = _lib.RowScatter()
    for n_dst, rows, base, msg in [(0, 16, 0, "n_dst"), (9, 16, 0, "n_dst"), (2, 15, 0, "multiples of 16"),
                                   (2, 16, 3, "multiples of 16")]:
        x.n_dst, x.slice_rows, x.row_base = n_dst, rows, base
        assert lib.llmx_attn_fwd_scatter(ctypes.byref(p), ctypes.byref(x), None) == 1  # LLMX_ERR_INVALID_ARGUMENT
        assert msg in lib.llmx_attn_last_error().decode()
    assert lib.llmx_ipc_alloc(1024, None, None) == 1  # LLMX_ERR_INVALID_ARGUMENT
    assert lib.llmx_ipc_open(None, None) == 1  # LLMX_ERR_INVALID_ARGUMENT
    assert lib.llmx_ipc_close(None) == 0
    assert lib.llmx_ipc_free(None) == 0
