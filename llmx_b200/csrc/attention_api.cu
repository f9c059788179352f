// C++ attention op over the C ABI (host code).
//
// llmx_single_mha_attention keeps the reference's checks and parameter
// mapping (src/cuda/attention/attention_api.cpp:14-72): contiguity of all
// four tensors, q [q_len, n_heads, D], k/v [kv_len, n_kv_heads, D], optional
// ALiBi slopes, causal, stream 0.  Failures throw std::runtime_error with the
// library's message.
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "llmx/cuda/attention/attention_api.h"
#include "llmx_attn.h"

namespace llmx {
namespace {

int32_t to_abi_dtype(ScalarType t) {
  switch (t) {
    case ScalarType::kFP32: return LLMX_FP32;
    case ScalarType::kFP16: return LLMX_FP16;
    case ScalarType::kBF16: return LLMX_BF16;
  }
  throw std::invalid_argument("llmx: unsupported dtype");
}

void check(bool ok, const char *msg) {
  if (!ok) throw std::runtime_error(std::string("llmx attention: ") + msg);
}

bool on_cuda(const Tensor &t) { return t.device().type == DeviceType::kCUDA; }

void check_devices(const Tensor &output, const Tensor &q, const Tensor &k, const Tensor &v,
                   const std::optional<Tensor> &alibi_slopes) {
  check(on_cuda(output) && on_cuda(q) && on_cuda(k) && on_cuda(v) &&
            (!alibi_slopes.has_value() || on_cuda(*alibi_slopes)),
        "tensors (and alibi_slopes) must be CUDA tensors");
}

void check_status(llmx_status s) {
  if (s != LLMX_OK)
    throw std::runtime_error(std::string("llmx attention: ") + llmx_status_string(s) + ": " +
                             llmx_attn_last_error());
}

// Grow-only split-KV scratch per device, owned by this wrapper (the C ABI
// itself never allocates).  Calls on different streams of one device share
// it, so they must not overlap; the reference is single-stream anyway.
struct Scratch {
  std::mutex mu;
  std::unordered_map<int, std::pair<void *, size_t>> by_device;
  void *get(int dev, size_t bytes) {
    std::lock_guard<std::mutex> lk(mu);
    auto &slot = by_device[dev];
    if (slot.second >= bytes) return slot.first;
    if (slot.first) cudaFree(slot.first);
    slot = {nullptr, 0};
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) throw std::runtime_error("llmx attention: workspace cudaMalloc failed");
    slot = {p, bytes};
    return p;
  }
};
Scratch &scratch() {
  static Scratch *s = new Scratch();  // never destroyed: may outlive the CUDA context at exit
  return *s;
}

}  // namespace

void llmx_single_mha_attention(Tensor &output, const Tensor &q, const Tensor &k, const Tensor &v,
                               const std::optional<Tensor> &alibi_slopes, float sm_scale,
                               int sliding_window, float logits_soft_cap) {
  check(output.contiguous() && q.contiguous() && k.contiguous() && v.contiguous(),
        "tensors must be contiguous");
  check(q.ndim() == 3 && k.ndim() == 3 && v.ndim() == 3 && output.ndim() == 3,
        "q, k, v, output must be 3-D [seq, heads, head_dim]");
  check_devices(output, q, k, v, alibi_slopes);
  check(q.dtype() == k.dtype() && q.dtype() == v.dtype() && q.dtype() == output.dtype(),
        "q, k, v, output must share a dtype");
  if (alibi_slopes.has_value())
    check(alibi_slopes->dtype() == ScalarType::kFP32 && alibi_slopes->numel() == size_t(q.dim(1)),
          "alibi_slopes must be fp32 [n_heads]");
  // Same request as llmx_single_mha_attention_c, but through the path that
  // hands the library its workspace (split-KV decode, prefill work queue).
  MHAOptions opts;
  opts.sliding_window = sliding_window;
  opts.logits_soft_cap = logits_soft_cap;
  llmx_mha_attention(output, q, k, v, alibi_slopes, sm_scale, opts);
}

void llmx_mha_attention(Tensor &output, const Tensor &q, const Tensor &k, const Tensor &v,
                        const std::optional<Tensor> &alibi_slopes, float sm_scale, const MHAOptions &opts) {
  check(output.contiguous() && q.contiguous() && k.contiguous() && v.contiguous(),
        "tensors must be contiguous");
  const bool three = q.ndim() == 3;
  check((three && k.ndim() == 3 && v.ndim() == 3 && output.ndim() == 3) ||
            (q.ndim() == 4 && k.ndim() == 4 && v.ndim() == 4 && output.ndim() == 4),
        "tensors must all be 3-D [S, H, D] or all 4-D [B, S, H, D]");
  check_devices(output, q, k, v, alibi_slopes);
  const int o = three ? 1 : 0;
  llmx_attn_params p;
  llmx_attn_params_init(&p);
  p.dtype = to_abi_dtype(q.dtype());
  p.batch = three ? 1 : q.dim(0);
  p.max_q_len = q.dim(1 - o);
  p.n_heads = q.dim(2 - o);
  p.head_dim = q.dim(3 - o);
  p.max_kv_len = k.dim(1 - o);
  p.n_kv_heads = k.dim(2 - o);
  p.q = q.const_data_ptr();
  p.k = k.const_data_ptr();
  p.v = v.const_data_ptr();
  p.o = output.data_ptr();
  llmx_attn_set_contiguous_strides(&p);
  if (alibi_slopes.has_value())
    check(alibi_slopes->dtype() == ScalarType::kFP32 && alibi_slopes->numel() == size_t(p.n_heads),
          "alibi_slopes must be fp32 [n_heads]");
  p.alibi_slopes = alibi_slopes.has_value() ? alibi_slopes->const_data_ptr<float>() : nullptr;
  p.sm_scale = sm_scale;
  p.causal = opts.causal ? 1 : 0;
  p.sliding_window = opts.sliding_window;
  p.logits_soft_cap = opts.logits_soft_cap;
  p.q_lens = opts.q_lens;
  p.kv_lens = opts.kv_lens;
  p.lse = opts.lse;
  size_t ws = 0;
  check_status(llmx_attn_workspace_size(&p, &ws));
  if (ws > 0) {
    int dev = 0;
    check(cudaGetDevice(&dev) == cudaSuccess, "no CUDA device");
    p.workspace = scratch().get(dev, ws);
    p.workspace_bytes = ws;
  }
  check_status(llmx_attn_fwd(&p, opts.stream));
}

}  // namespace llmx
