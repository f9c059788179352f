// Operator registry (host code): the executor, the conversion operators and
// the attention operator behind include/llmx/ops.h.
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "llmx/ops.h"

namespace llmx {
namespace {

void require(bool ok, const std::string &msg) {
  if (!ok) throw std::runtime_error("llmx ops: " + msg);
}

Tensor *get(TensorDict &data, const char *name) {
  auto it = data.find(name);
  require(it != data.end() && it->second != nullptr, std::string("missing tensor \"") + name + "\"");
  return it->second;
}

template <typename T>
T param_or(const Parameters &params, const char *name, T fallback) {
  auto it = params.find(name);
  if (it == params.end()) return fallback;
  try {
    return std::any_cast<T>(it->second);
  } catch (const std::bad_any_cast &) {
    throw std::runtime_error(std::string("llmx ops: parameter \"") + name + "\" has the wrong type");
  }
}

template <typename T>
T param(const Parameters &params, const char *name) {
  require(params.count(name) != 0, std::string("missing parameter \"") + name + "\"");
  return param_or<T>(params, name, T{});
}

bool is_half(ScalarType t) { return t == ScalarType::kFP16 || t == ScalarType::kBF16; }

}  // namespace

// ---- conversion ----------------------------------------------------------

void CudaConvert::pre_run(TensorDict &data, const Parameters &) {
  Tensor *in = get(data, "input");
  Tensor *out = get(data, "output");
  out->dtype(to);
  out->resize(in->dims());
  out->allocate();
}

void CudaConvert::run(TensorDict &data, const Parameters &) {
  Tensor *in = get(data, "input");
  Tensor *out = get(data, "output");
  require(in->contiguous(), "conversion input must be contiguous");
  llmx_copy(in->dtype(), out->dtype(), in->const_data_ptr(), out->data_ptr(), in->numel());
}

// ---- attention -----------------------------------------------------------

void CudaAttentionHalf::pre_run(TensorDict &data, const Parameters &) {
  Tensor *q = get(data, "query");
  Tensor *k = get(data, "key");
  Tensor *v = get(data, "value");
  Tensor *out = get(data, "output");
  const int nd = q->ndim();
  require(nd == 3 || nd == 4, "query must be [q_len, n_heads, head_dim] or [batch, q_len, n_heads, head_dim]");
  require(k->ndim() == nd && v->ndim() == nd, "key and value must have the query's rank");
  require(q->dtype() == k->dtype() && q->dtype() == v->dtype(), "query, key and value must share a dtype");
  require(is_half(q->dtype()) || q->dtype() == ScalarType::kFP32, "dtype must be fp16, bf16 or fp32");
  require(q->dim(nd - 1) == k->dim(nd - 1) && q->dim(nd - 1) == v->dim(nd - 1), "head_dim mismatch");
  out->dtype(q->dtype());
  out->resize(q->dims());
  out->allocate();
}

void CudaAttentionHalf::run(TensorDict &data, const Parameters &params) {
  Tensor *q = get(data, "query");
  Tensor *k = get(data, "key");
  Tensor *v = get(data, "value");
  Tensor *out = get(data, "output");
  std::optional<Tensor> slopes = param<std::optional<Tensor>>(params, "alibi_slopes");
  if (slopes.has_value() && slopes->device() != out->device()) {
    // A parameter is not moved by the executor; a host copy of the slopes
    // would be dereferenced by the kernel, so move a private copy.
    Tensor moved = *slopes;
    moved.to_device(out->device());
    slopes = moved;
  }
  MHAOptions o;
  o.causal = param_or<bool>(params, "causal", true);
  o.sliding_window = param<int>(params, "sliding_window");
  o.logits_soft_cap = param<float>(params, "logits_soft_cap");
  o.q_lens = param_or<const int *>(params, "q_lens", nullptr);
  o.kv_lens = param_or<const int *>(params, "kv_lens", nullptr);
  Tensor *lse = param_or<Tensor *>(params, "lse", nullptr);
  if (lse != nullptr) {
    require(lse->dtype() == ScalarType::kFP32 && lse->device() == out->device() && lse->contiguous(),
            "lse must be a contiguous fp32 tensor on the output's device");
    const int nd = q->ndim();
    const size_t rows = size_t(nd == 4 ? q->dim(0) : 1) * q->dim(nd - 2) * q->dim(nd - 3);
    require(lse->numel() >= rows, "lse must hold batch * n_heads * q_len values");
    o.lse = lse->data_ptr<float>();
  }
  o.stream = param_or<void *>(params, "stream", nullptr);
  const float sm_scale = param<float>(params, "sm_scale");
  llmx_mha_attention(*out, *q, *k, *v, slopes, sm_scale, o);
}

// ---- executor ------------------------------------------------------------

CudaExecutorImpl::CudaExecutorImpl(int id) : ExecutorImpl(Device(DeviceType::kCUDA, id)) {
  ops["to_fp32_op"] = std::make_unique<CudaToFloat32>();
  ops["to_fp16_op"] = std::make_unique<CudaToFloat16>();
  ops["to_bf16_op"] = std::make_unique<CudaToBFloat16>();
  ops["attention_haft_op"] = std::make_unique<CudaAttentionHalf>();
}

struct Executor::State {
  std::mutex mu;
  std::vector<std::unique_ptr<ExecutorImpl>> devices;  // index = CUDA ordinal, built on first use
  int n_devices = -1;

  // Every CUDA device's executor, built on first use.  Caller holds mu.
  void ensure() {
    if (n_devices >= 0) return;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    n_devices = n;
    for (int i = 0; i < n; ++i) devices.push_back(std::make_unique<CudaExecutorImpl>(i));
  }
};

Executor::Executor() : state_(std::make_unique<State>()) {}
Executor::~Executor() = default;

bool Executor::can_run(const std::string &op_name) const {
  std::lock_guard<std::mutex> lk(state_->mu);
  state_->ensure();
  for (auto &d : state_->devices)
    if (d->can_run(op_name)) return true;
  return false;
}

void Executor::register_op(int device_id, const std::string &op_name, std::unique_ptr<OperatorBase> op) {
  std::lock_guard<std::mutex> lk(state_->mu);
  state_->ensure();
  require(device_id >= 0 && device_id < state_->n_devices, "register_op: no such CUDA device");
  state_->devices[device_id]->ops[op_name] = std::move(op);
}

void Executor::run(const std::string &op_name, TensorDict data, const Parameters &params) {
  ExecutorImpl *exe = nullptr;
  {
    std::lock_guard<std::mutex> lk(state_->mu);
    state_->ensure();
    for (auto &d : state_->devices)
      if (d->can_run(op_name)) {
        exe = d.get();
        break;
      }
  }
  require(exe != nullptr, "could not find a device to execute operator " + op_name);
  for (auto &kv : data) {
    if (kv.second == nullptr) continue;
    if (kv.first == "output") {
      kv.second->to_device(exe->device, false);
    } else {
      require(kv.second->is_valid(), "input tensor \"" + kv.first + "\" holds no storage");
      kv.second->to_device(exe->device);
    }
  }
  int prev = 0;
  require(cudaGetDevice(&prev) == cudaSuccess, "cudaGetDevice failed");
  require(cudaSetDevice(exe->device.id) == cudaSuccess, "cudaSetDevice failed");
  struct Restore {
    int dev;
    ~Restore() { cudaSetDevice(dev); }
  } restore{prev};
  OperatorBase &op = exe->op(op_name);
  op.pre_run(data, params);
  op.run(data, params);
  op.post_run(data, params);
}

Executor *get_op_executor() {
  static Executor *e = new Executor();  // never destroyed: may outlive the CUDA context at exit
  return e;
}

}  // namespace llmx
