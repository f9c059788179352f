// llmx's operator registry: named operators run through a process-wide
// executor, as the reference's include/llmx/ops.h:14-229 does.
//
// Kept from the reference, so its callers compile unchanged:
//  * TensorDict / Parameters / OperatorBase (pre_run, run, post_run);
//  * the CUDA operators under their registered names "to_fp32_op",
//    "to_fp16_op", "to_bf16_op" and "attention_haft_op" (ops.h:148-155), and
//    the free functions to_fp32 / to_fp16 / to_bf16;
//  * Executor::run moves "output" to the executing device without copying
//    and every other (valid) tensor with a copy (ops.h:176-200), then calls
//    pre_run, run and post_run.
// Changed:
//  * get_op_executor() is one instance per process, defined in the library
//    (the reference's header-static gives one per translation unit);
//  * to_fp16 looks up "to_fp16_op" (the reference asks for "tto_fp16_op",
//    ops.h:224, which no executor registers, so its to_fp16 always fails);
//  * "attention_haft_op" also takes 4-D [B, S, H, D] tensors, fp32, and the
//    optional parameters "causal" (bool), "q_lens" / "kv_lens" (const int *,
//    device int32 [B]), "lse" (Tensor *, fp32 [B, H, S_q]) and "stream"
//    (void *, a cudaStream_t) -- the batched / padded / non-causal forms of
//    llmx_mha_attention;
//  * errors throw std::runtime_error instead of LLMX_CHECK's terminate;
//  * an executor for a device is built on first use, not for every device at
//    start-up.
#pragma once

#include <any>
#include <memory>
#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "llmx/cuda/attention/attention_api.h"
#include "llmx/tensor.h"

namespace llmx {

using TensorDict = std::unordered_map<std::string, Tensor *>;
using Parameters = std::unordered_map<std::string, std::any>;

struct OperatorBase {
  virtual ~OperatorBase() = default;
  virtual void pre_run(TensorDict &data, const Parameters &params) {}
  virtual void post_run(TensorDict &data, const Parameters &params) {}
  virtual void run(TensorDict &data, const Parameters &params) = 0;
};

// "input" -> "output" in the operator's dtype; output resized to the input's
// dims and (re)allocated on the device (ops.h:25-74).
struct CudaConvert : public OperatorBase {
  explicit CudaConvert(ScalarType to) : to(to) {}
  void pre_run(TensorDict &data, const Parameters &params) override;
  void run(TensorDict &data, const Parameters &params) override;
  ScalarType to;
};
struct CudaToFloat32 : public CudaConvert {
  CudaToFloat32() : CudaConvert(ScalarType::kFP32) {}
};
struct CudaToFloat16 : public CudaConvert {
  CudaToFloat16() : CudaConvert(ScalarType::kFP16) {}
};
struct CudaToBFloat16 : public CudaConvert {
  CudaToBFloat16() : CudaConvert(ScalarType::kBF16) {}
};

// "query" / "key" / "value" -> "output" (ops.h:76-113), parameters
// "alibi_slopes" (std::optional<Tensor>), "sm_scale" (float),
// "sliding_window" (int), "logits_soft_cap" (float), plus the optional
// extensions listed at the top of this file.
struct CudaAttentionHalf : public OperatorBase {
  void pre_run(TensorDict &data, const Parameters &params) override;
  void run(TensorDict &data, const Parameters &params) override;
};

// The operators of one device.
struct ExecutorImpl {
  explicit ExecutorImpl(Device device) : device(device) {}
  virtual ~ExecutorImpl() = default;
  bool can_run(const std::string &op_name) const { return ops.count(op_name) != 0; }
  OperatorBase &op(const std::string &op_name) { return *ops.at(op_name); }

  std::unordered_map<std::string, std::unique_ptr<OperatorBase>> ops;
  Device device;
};

struct CudaExecutorImpl : public ExecutorImpl {
  explicit CudaExecutorImpl(int id);
};

class Executor {
 public:
  Executor();
  ~Executor();
  Executor(const Executor &) = delete;
  Executor &operator=(const Executor &) = delete;

  // Runs `op_name` on the first device whose executor has it (device order:
  // CUDA 0, 1, ...), after moving the tensors there.  Throws when no device
  // has the operator or an input tensor holds no storage.
  void run(const std::string &op_name, TensorDict data, const Parameters &params);
  bool can_run(const std::string &op_name) const;
  // Adds (or replaces) an operator on CUDA device `device_id`.
  void register_op(int device_id, const std::string &op_name, std::unique_ptr<OperatorBase> op);

 private:
  struct State;
  std::unique_ptr<State> state_;
};

Executor *get_op_executor();

inline void to_fp32(Tensor &output, const Tensor &input) {
  get_op_executor()->run("to_fp32_op", {{"input", const_cast<Tensor *>(&input)}, {"output", &output}}, {});
}
inline void to_fp16(Tensor &output, const Tensor &input) {
  get_op_executor()->run("to_fp16_op", {{"input", const_cast<Tensor *>(&input)}, {"output", &output}}, {});
}
inline void to_bf16(Tensor &output, const Tensor &input) {
  get_op_executor()->run("to_bf16_op", {{"input", const_cast<Tensor *>(&input)}, {"output", &output}}, {});
}

// Convenience form of "attention_haft_op": output is resized and allocated
// like q.  `extra` may carry the optional parameters listed above.
inline void attention(Tensor &output, const Tensor &q, const Tensor &k, const Tensor &v,
                      const std::optional<Tensor> &alibi_slopes, float sm_scale, int sliding_window = -1,
                      float logits_soft_cap = 0.f, Parameters extra = {}) {
  extra["alibi_slopes"] = alibi_slopes;
  extra["sm_scale"] = sm_scale;
  extra["sliding_window"] = sliding_window;
  extra["logits_soft_cap"] = logits_soft_cap;
  get_op_executor()->run("attention_haft_op",
                         {{"query", const_cast<Tensor *>(&q)},
                          {"key", const_cast<Tensor *>(&k)},
                          {"value", const_cast<Tensor *>(&v)},
                          {"output", &output}},
                         extra);
}

}  // namespace llmx
