// Torch binding of llmx's attention op: the Python function the reference
// exposes from csrc/llmx_bind.cpp:35-78,
//
//   single_mha_attention_half(output, q, k, v, sm_scale,
//                             sliding_window=-1, logits_soft_cap=0.0)
//
// with the same name, argument order, defaults and TORCH_CHECK conditions
// (3-D tensors, one dtype, CUDA tensors on one device, n_heads divisible by
// n_kv_heads, matching head_dim; llmx_bind.cpp:41-58), built as a torch
// extension over the C ABI in llmx_attn.h.  Differences, all additive:
//  * keyword arguments alibi_slopes, causal, q_lens, kv_lens, lse (the
//    reference always passes no slopes and runs causal only,
//    llmx_bind.cpp:69-71);
//  * 4-D [batch, seq, heads, head_dim] tensors and fp32;
//  * strided q / k / v / output (unit stride on head_dim) are passed as they
//    are instead of being made contiguous;
//  * the work runs on torch's current CUDA stream, not stream 0;
//  * split-KV decode scratch comes from torch's caching allocator;
//  * algo (force one kernel family) and kv_offset / kv_total (a shard of a
//    sequence's keys at its global positions) as in llmx_attn_params.
// Library failures raise llmx_b200.LlmxError (a RuntimeError) carrying the
// llmx_status and the library's message.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <optional>
#include <string>

#include "llmx_attn.h"

namespace py = pybind11;

namespace {

int32_t llmx_dtype_of(const torch::Tensor &t) {
  switch (t.scalar_type()) {
    case torch::kFloat: return LLMX_FP32;
    case torch::kHalf: return LLMX_FP16;
    case torch::kBFloat16: return LLMX_BF16;
    default:
      TORCH_CHECK(false, "llmx: unsupported dtype ", t.scalar_type(),
                  ". Only float16, bfloat16, float32 are supported.");
  }
  return -1;
}

void set_strides(int64_t (&dst)[3], const torch::Tensor &t, bool four) {
  dst[0] = four ? t.stride(0) : 0;
  dst[1] = t.stride(four ? 1 : 0);
  dst[2] = t.stride(four ? 2 : 1);
}

// A failing llmx_status, raised to Python as llmx_b200.LlmxError(status, message).
struct StatusError {
  int status;
  std::string message;
};

void check_status(llmx_status s) {
  if (s != LLMX_OK) throw StatusError{(int)s, llmx_attn_last_error()};
}

int32_t algo_code(const std::string &name) {
  if (name == "auto") return LLMX_ALGO_AUTO;
  if (name == "simt") return LLMX_ALGO_SIMT;
  if (name == "decode") return LLMX_ALGO_DECODE;
  if (name == "tcgen05") return LLMX_ALGO_TCGEN05;
  TORCH_CHECK(false, "algo must be one of auto, simt, decode, tcgen05");
  return 0;
}

}  // namespace

void single_mha_attention_half(torch::Tensor output, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                               double sm_scale, int64_t sliding_window, double logits_soft_cap,
                               std::optional<torch::Tensor> alibi_slopes, bool causal,
                               std::optional<torch::Tensor> q_lens, std::optional<torch::Tensor> kv_lens,
                               std::optional<torch::Tensor> lse, const std::string &algo, int64_t kv_offset,
                               int64_t kv_total) {
  const int64_t nd = q.dim();
  TORCH_CHECK((nd == 3 || nd == 4) && k.dim() == nd && v.dim() == nd && output.dim() == nd,
              "q, k, v must be 3-D: [seq, heads, head_dim] (or all 4-D: [batch, seq, heads, head_dim])");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
              "q, k, v must have the same dtype");
  TORCH_CHECK(output.scalar_type() == q.scalar_type(), "output must have the dtype of q");
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && output.is_cuda(), "q, k, v must be CUDA tensors");
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device() && q.device() == output.device(),
              "q, k, v must be on the same device");
  const bool four = nd == 4;
  const int64_t B = four ? q.size(0) : 1;
  const int64_t Sq = q.size(nd - 3), H = q.size(nd - 2), D = q.size(nd - 1);
  const int64_t Skv = k.size(nd - 3), Hkv = k.size(nd - 2);
  TORCH_CHECK(H % Hkv == 0, "n_heads (", H, ") must be divisible by n_kv_heads (", Hkv, ")");
  TORCH_CHECK(q.size(nd - 1) == k.size(nd - 1) && q.size(nd - 1) == v.size(nd - 1),
              "head_dim must match across q, k, v");
  TORCH_CHECK(k.sizes() == v.sizes(), "k and v must have the same shape");
  TORCH_CHECK(output.sizes() == q.sizes(), "output must have the shape of q");
  TORCH_CHECK(!four || (k.size(0) == B && v.size(0) == B), "batch sizes must match");
  // Rows with a unit head_dim stride are taken as they are (the reference
  // makes every input contiguous, llmx_bind.cpp:60-62).
  if (q.stride(-1) != 1) q = q.contiguous();
  if (k.stride(-1) != 1) k = k.contiguous();
  if (v.stride(-1) != 1) v = v.contiguous();
  TORCH_CHECK(output.stride(-1) == 1, "output must have a unit stride on head_dim");

  const c10::cuda::CUDAGuard guard(q.device());
  llmx_attn_params p;
  check_status(llmx_attn_params_init(&p));
  p.dtype = llmx_dtype_of(q);
  p.batch = (int32_t)B;
  p.n_heads = (int32_t)H;
  p.n_kv_heads = (int32_t)Hkv;
  p.head_dim = (int32_t)D;
  p.max_q_len = (int32_t)Sq;
  p.max_kv_len = (int32_t)Skv;
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.o = output.data_ptr();
  set_strides(p.q_stride, q, four);
  set_strides(p.k_stride, k, four);
  set_strides(p.v_stride, v, four);
  set_strides(p.o_stride, output, four);
  torch::Tensor slopes, ql, kl;
  if (alibi_slopes.has_value()) {
    TORCH_CHECK(alibi_slopes->is_cuda() && alibi_slopes->device() == q.device(), "alibi_slopes must be on q's device");
    slopes = alibi_slopes->to(torch::kFloat).contiguous();
    TORCH_CHECK(slopes.numel() == H, "alibi_slopes must have n_heads elements");
    p.alibi_slopes = slopes.data_ptr<float>();
  }
  if (q_lens.has_value()) {
    TORCH_CHECK(q_lens->is_cuda() && q_lens->device() == q.device(), "q_lens must be on q's device");
    ql = q_lens->to(torch::kInt).contiguous();
    TORCH_CHECK(ql.numel() == B, "q_lens must have batch elements");
    p.q_lens = ql.data_ptr<int32_t>();
  }
  if (kv_lens.has_value()) {
    TORCH_CHECK(kv_lens->is_cuda() && kv_lens->device() == q.device(), "kv_lens must be on q's device");
    kl = kv_lens->to(torch::kInt).contiguous();
    TORCH_CHECK(kl.numel() == B, "kv_lens must have batch elements");
    p.kv_lens = kl.data_ptr<int32_t>();
  }
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == torch::kFloat && lse->is_contiguous() && lse->device() == q.device() &&
                    lse->dim() == 3 && lse->size(0) == B && lse->size(1) == H && lse->size(2) == Sq,
                "lse must be contiguous fp32 [batch, n_heads, max_q_len] on q's device");
    p.lse = lse->data_ptr<float>();
  }
  p.sm_scale = (float)sm_scale;
  p.causal = causal ? 1 : 0;
  p.sliding_window = (int32_t)sliding_window;
  p.logits_soft_cap = (float)logits_soft_cap;
  p.algo = algo_code(algo);
  p.kv_offset = (int32_t)kv_offset;
  p.kv_total = (int32_t)kv_total;
  size_t ws_bytes = 0;
  check_status(llmx_attn_workspace_size(&p, &ws_bytes));
  torch::Tensor ws;
  if (ws_bytes > 0) {
    ws = torch::empty({(int64_t)ws_bytes}, q.options().dtype(torch::kByte));
    p.workspace = ws.data_ptr();
    p.workspace_bytes = ws_bytes;
  }
  check_status(llmx_attn_fwd(&p, at::cuda::getCurrentCUDAStream(q.device().index()).stream()));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "llmx attention op on B200 (sm_100a): torch binding over libllmx_attn.so";
  static py::object error_cls = py::module_::import("llmx_b200._lib").attr("LlmxError");
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const StatusError &e) {
      py::object err = error_cls(e.status, e.message);
      PyErr_SetObject(error_cls.ptr(), err.ptr());
    }
  });
  m.def("single_mha_attention_half", &single_mha_attention_half, py::arg("output"), py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("sm_scale"), py::arg("sliding_window") = -1, py::arg("logits_soft_cap") = 0.0,
        py::kw_only(), py::arg("alibi_slopes") = py::none(), py::arg("causal") = true,
        py::arg("q_lens") = py::none(), py::arg("kv_lens") = py::none(), py::arg("lse") = py::none(),
        py::arg("algo") = "auto", py::arg("kv_offset") = 0, py::arg("kv_total") = 0);
  m.def("abi_version", [] { return llmx_attn_abi_version(); });
}
