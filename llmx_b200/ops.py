"""Torch-facing attention op: the reference binding's surface over the C ABI.

``single_mha_attention_half`` keeps the name, argument order and defaults of
the reference's pybind11 function (csrc/llmx_bind.cpp:35-78):

    single_mha_attention_half(output, q, k, v, sm_scale,
                              sliding_window=-1, logits_soft_cap=0.0)

and its checks (llmx_bind.cpp:41-58: 3-D tensors, one dtype, CUDA, one
device, n_heads divisible by n_kv_heads, matching head_dim), raising
RuntimeError where the reference raises through TORCH_CHECK.  It adds the
extended request as keyword arguments: ``alibi_slopes`` (the reference
binding always passes nullopt, llmx_bind.cpp:69-71), ``causal``, ``q_lens``
/ ``kv_lens`` (padding), ``lse``, ``kv_offset`` / ``kv_total`` (key shards),
4-D [B, S, H, D] tensors, fp32, and it runs on torch's current stream
instead of stream 0.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_TORCH_DTYPE = {torch.float32: "fp32", torch.float16: "fp16", torch.bfloat16: "bf16"}


def _req(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _strides(t: torch.Tensor, four: bool):
    st = t.stride()
    return (st[0], st[1], st[2]) if four else (0, st[0], st[1])


def build_params(
    output: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    sm_scale: float,
    sliding_window: int = -1,
    logits_soft_cap: float = 0.0,
    *,
    alibi_slopes: Optional[torch.Tensor] = None,
    causal: bool = True,
    q_lens: Optional[torch.Tensor] = None,
    kv_lens: Optional[torch.Tensor] = None,
    lse: Optional[torch.Tensor] = None,
    algo: str = "auto",
    kv_offset: int = 0,
    kv_total: int = 0,
):
    """Validates torch tensors and returns (AttnParams, tensors to keep alive)."""
    nd = q.dim()
    _req(nd in (3, 4) and k.dim() == nd and v.dim() == nd and output.dim() == nd,
         "q, k, v must be 3-D: [seq, heads, head_dim] (or all 4-D: [batch, seq, heads, head_dim])")
    _req(q.dtype == k.dtype and q.dtype == v.dtype, "q, k, v must have the same dtype")
    _req(q.dtype in _TORCH_DTYPE, "Only float16, bfloat16 and float32 are supported")
    _req(output.dtype == q.dtype, "output must have the dtype of q")
    _req(q.is_cuda and k.is_cuda and v.is_cuda and output.is_cuda, "q, k, v must be CUDA tensors")
    _req(q.device == k.device == v.device == output.device, "q, k, v must be on the same device")
    four = nd == 4
    B = q.shape[0] if four else 1
    _req(k.shape[0] == B and v.shape[0] == B and output.shape[0] == B or not four, "batch sizes must match")
    Sq, H, D = q.shape[-3], q.shape[-2], q.shape[-1]
    Skv, Hkv = k.shape[-3], k.shape[-2]
    _req(H % Hkv == 0, f"n_heads ({H}) must be divisible by n_kv_heads ({Hkv})")
    _req(q.shape[-1] == k.shape[-1] == v.shape[-1], "head_dim must match across q, k, v")
    _req(tuple(v.shape) == tuple(k.shape), "k and v must have the same shape")
    _req(tuple(output.shape) == tuple(q.shape), "output must have the shape of q")
    # The reference makes q, k, v contiguous (llmx_bind.cpp:60-62); rows with a
    # unit inner stride are passed as they are, others are copied.
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    _req(output.stride(-1) == 1, "output must have a unit stride on head_dim")
    keep = [q, k, v, output]

    p = _lib.AttnParams()
    _lib.check(_lib.load().llmx_attn_params_init(ctypes.byref(p)))
    p.dtype = _lib.DTYPE[_TORCH_DTYPE[q.dtype]]
    p.batch, p.n_heads, p.n_kv_heads, p.head_dim = B, H, Hkv, D
    p.max_q_len, p.max_kv_len = Sq, Skv
    p.algo = _lib.ALGO[algo]
    p.q, p.k, p.v, p.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), output.data_ptr()
    for name, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", output)):
        getattr(p, name)[:] = _strides(t, four)
    if alibi_slopes is not None:
        _req(alibi_slopes.is_cuda and alibi_slopes.device == q.device, "alibi_slopes must be on q's device")
        a = alibi_slopes.to(torch.float32).contiguous()
        _req(a.numel() == H, "alibi_slopes must have n_heads elements")
        keep.append(a)
        p.alibi_slopes = a.data_ptr()
    for name, lens in (("q_lens", q_lens), ("kv_lens", kv_lens)):
        if lens is not None:
            _req(lens.is_cuda and lens.device == q.device, f"{name} must be on q's device")
            t = lens.to(torch.int32).contiguous()
            _req(t.numel() == B, f"{name} must have batch elements")
            keep.append(t)
            setattr(p, name, t.data_ptr())
    if lse is not None:
        _req(lse.dtype == torch.float32 and lse.is_contiguous() and tuple(lse.shape) == (B, H, Sq),
             "lse must be contiguous fp32 [batch, n_heads, max_q_len]")
        _req(lse.device == q.device, "lse must be on q's device")
        p.lse = lse.data_ptr()
    p.sm_scale = float(sm_scale)
    p.kv_offset, p.kv_total = int(kv_offset), int(kv_total)
    p.causal = 1 if causal else 0
    p.sliding_window = int(sliding_window)
    p.logits_soft_cap = float(logits_soft_cap)
    return p, keep


def _run(p, device: torch.device, keep) -> None:
    lib = _lib.load()
    with torch.cuda.device(device):
        ws = ctypes.c_size_t(0)
        _lib.check(lib.llmx_attn_workspace_size(ctypes.byref(p), ctypes.byref(ws)))
        if ws.value:
            # torch's caching allocator: stream-ordered, no cudaMalloc per call.
            buf = torch.empty(ws.value, dtype=torch.uint8, device=device)
            keep.append(buf)
            p.workspace, p.workspace_bytes = buf.data_ptr(), ws.value
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(lib.llmx_attn_fwd(ctypes.byref(p), ctypes.c_void_p(stream)))


_EXT = None


def _extension():
    """The C++ torch binding (llmx_b200.llmx_bind, built by
    ``python -m llmx_b200.build``), or None when it has not been built."""
    global _EXT
    if _EXT is None:
        try:
            from . import llmx_bind

            _EXT = llmx_bind
        except ImportError:
            _EXT = False
    return _EXT or None


def single_mha_attention_half(
    output: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    sm_scale: float,
    sliding_window: int = -1,
    logits_soft_cap: float = 0.0,
    *,
    alibi_slopes: Optional[torch.Tensor] = None,
    causal: bool = True,
    q_lens: Optional[torch.Tensor] = None,
    kv_lens: Optional[torch.Tensor] = None,
    lse: Optional[torch.Tensor] = None,
    algo: str = "auto",
    kv_offset: int = 0,
    kv_total: int = 0,
) -> None:
    """Writes attention(q, k, v) into ``output`` (see the module docstring).

    ``kv_offset`` / ``kv_total`` describe a shard of a sequence's keys: local
    key j sits at global position kv_offset + j and the causal / window
    diagonal uses the full key length kv_total (0: the local length).

    Runs through the C++ torch binding (llmx_b200.llmx_bind: the checks and
    the C-ABI call in C++, a few microseconds of host time) when it is built,
    else through ctypes (``single_mha_attention_half_ctypes``); both call
    the same library entry points with the same request."""
    ext = _extension()
    if ext is not None:
        ext.single_mha_attention_half(output, q, k, v, float(sm_scale), int(sliding_window), float(logits_soft_cap),
                                      alibi_slopes=alibi_slopes, causal=bool(causal), q_lens=q_lens, kv_lens=kv_lens,
                                      lse=lse, algo=algo, kv_offset=int(kv_offset), kv_total=int(kv_total))
        return
    single_mha_attention_half_ctypes(output, q, k, v, sm_scale, sliding_window, logits_soft_cap,
                                     alibi_slopes=alibi_slopes, causal=causal, q_lens=q_lens, kv_lens=kv_lens,
                                     lse=lse, algo=algo, kv_offset=kv_offset, kv_total=kv_total)


def single_mha_attention_half_ctypes(output, q, k, v, sm_scale, sliding_window=-1, logits_soft_cap=0.0, **kw):
    """The same op through ctypes over the C ABI (no compiled binding needed)."""
    p, keep = build_params(output, q, k, v, sm_scale, sliding_window, logits_soft_cap, **kw)
    _run(p, q.device, keep)


def attention(q, k, v, sm_scale=None, **kw) -> torch.Tensor:
    """Allocating convenience form: returns a new output tensor."""
    out = torch.empty_like(q)
    if sm_scale is None:
        sm_scale = q.shape[-1] ** -0.5
    single_mha_attention_half(out, q, k, v, sm_scale, **kw)
    return out


def selected_algo(output, q, k, v, sm_scale, **kw) -> str:
    """Name of the kernel family the library would run for this request."""
    p, _ = build_params(output, q, k, v, sm_scale, **kw)
    out = ctypes.c_int32(0)
    _lib.check(_lib.load().llmx_attn_select_algo(ctypes.byref(p), ctypes.byref(out)))
    return _lib.ALGO_NAMES[out.value]


def device_status(device: int = 0, clear: bool = True) -> None:
    """Raises LlmxError if a kernel on `device` gave up on a bounded wait."""
    _lib.check(_lib.load().llmx_attn_device_status(int(device), 1 if clear else 0))


def convert(x: torch.Tensor, dtype: torch.dtype, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Element-type conversion between fp32, fp16 and bf16 on the library's
    kernel (the to_fp32 / to_fp16 / to_bf16 ops, include/llmx/ops.h:25-74 and
    src/scalar.cu:33-46 in the reference), round to nearest even, on torch's
    current stream.  ``x`` is a contiguous CUDA tensor; ``out`` (optional) a
    contiguous CUDA tensor of ``dtype`` with as many elements."""
    _req(x.is_cuda, "convert: input must be a CUDA tensor")
    _req(x.dtype in _TORCH_DTYPE and dtype in _TORCH_DTYPE, "convert: dtypes must be fp32, fp16 or bf16")
    _req(x.is_contiguous(), "convert: input must be contiguous")
    if out is None:
        out = torch.empty(x.shape, dtype=dtype, device=x.device)
    _req(out.is_cuda and out.device == x.device and out.dtype == dtype and out.is_contiguous()
         and out.numel() == x.numel(), "convert: out must be a contiguous CUDA tensor of dtype with x's size")
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(_lib.load().llmx_convert(ctypes.c_void_p(x.data_ptr()), _lib.DTYPE[_TORCH_DTYPE[x.dtype]],
                                            ctypes.c_void_p(out.data_ptr()), _lib.DTYPE[_TORCH_DTYPE[dtype]],
                                            x.numel(), ctypes.c_void_p(stream)))
    return out
