// C ABI of the attention engine: validation, kernel selection and launch.
//
// Mirrors the reference host layer (src/cuda/attention/attention_api.cpp:14-72
// and MHAParams::normalize, params.h:35-50) with three differences:
//  * errors come back as llmx_status instead of LLMX_CHECK's terminate
//    (utility.h:76-143), with a per-thread message;
//  * device attributes are cached once per device (the reference queries
//    cudaGetDeviceProperties on every launch, single_mha_kernel.cuh:618-619);
//  * work goes to the caller's stream (the reference uses stream 0,
//    attention_api.cpp:55).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "llmx_attn.h"
#include "attn_internal.h"

namespace llmx_b200 {
namespace {

thread_local std::string g_last_error;

// One error word per device, OR-ed by kernels whose bounded waits expire.
__device__ unsigned int g_device_error_word;

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ok = false;
  int num_sms = 0;
  int major = 0, minor = 0;
  unsigned int *err = nullptr;
  std::string why;
};

DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

const DeviceInfo &device_info(int dev) {
  std::call_once(g_dev_once[dev], [dev] {
    DeviceInfo &d = g_dev[dev];
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
      d.why = "cudaGetDeviceProperties failed";
      return;
    }
    d.num_sms = prop.multiProcessorCount;
    d.major = prop.major;
    d.minor = prop.minor;
    if (prop.major != 10) {
      char buf[160];
      snprintf(buf, sizeof buf, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
               prop.major, prop.minor);
      d.why = buf;
      return;
    }
    void *addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_device_error_word) != cudaSuccess || addr == nullptr) {
      d.why = "cudaGetSymbolAddress(error word) failed";
      return;
    }
    d.err = static_cast<unsigned int *>(addr);
    d.ok = true;
  });
  return g_dev[dev];
}

llmx_status fail(llmx_status s, const std::string &msg) {
  g_last_error = msg;
  return s;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 16-byte vector access to rows of head_dim elements.
bool rows_vectorizable(const AttnArgs &a) {
  const int es = a.dtype == LLMX_FP32 ? 4 : 2;
  const int vec = 16 / es;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.o)) return false;
  if (a.D % vec) return false;
  for (int i = 0; i < 3; ++i) {
    if (a.qs[i] % vec || a.ks[i] % vec || a.vs[i] % vec || a.os[i] % vec) return false;
  }
  return true;
}

bool decode_supports(const AttnArgs &a) {
  return a.dtype != LLMX_FP32 && a.Sq == 1 && (a.D == 64 || a.D == 128 || a.D == 256) &&
         rows_vectorizable(a);
}

llmx_status validate(const llmx_attn_params *p, AttnArgs *a) {
  if (p == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "params is NULL");
  if (p->dtype < LLMX_FP32 || p->dtype > LLMX_BF16)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "dtype must be LLMX_FP32, LLMX_FP16 or LLMX_BF16");
  if (p->batch < 1 || p->n_heads < 1 || p->n_kv_heads < 1 || p->max_q_len < 1 || p->max_kv_len < 1)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "batch, heads and lengths must be >= 1");
  if (p->batch > 65535 || p->n_heads > 65535)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "batch and n_heads must be <= 65535");
  if (p->n_heads % p->n_kv_heads != 0)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "n_heads must be divisible by n_kv_heads");
  if (p->head_dim < 1 || p->head_dim > 256)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "head_dim must be in [1, 256]");
  if (!p->q || !p->k || !p->v || !p->o)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "q, k, v and o must be non-NULL");
  if (!std::isfinite(p->sm_scale)) return fail(LLMX_ERR_INVALID_ARGUMENT, "sm_scale must be finite");
  if (!std::isfinite(p->logits_soft_cap))
    return fail(LLMX_ERR_INVALID_ARGUMENT, "logits_soft_cap must be finite");
  if (p->algo < LLMX_ALGO_AUTO || p->algo > LLMX_ALGO_TCGEN05)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "unknown algo");
  if (p->kv_offset < 0 || p->kv_total < 0)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "kv_offset and kv_total must be >= 0");
  const int64_t *st[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t)
    for (int i = 0; i < 3; ++i)
      if (st[t][i] < 0) return fail(LLMX_ERR_INVALID_ARGUMENT, "strides must be >= 0");
  a->dtype = p->dtype;
  a->B = p->batch;
  a->H = p->n_heads;
  a->Hkv = p->n_kv_heads;
  a->D = p->head_dim;
  a->Sq = p->max_q_len;
  a->Skv = p->max_kv_len;
  a->group = p->n_heads / p->n_kv_heads;
  a->q = p->q;
  a->k = p->k;
  a->v = p->v;
  a->o = p->o;
  for (int i = 0; i < 3; ++i) {
    a->qs[i] = p->q_stride[i];
    a->ks[i] = p->k_stride[i];
    a->vs[i] = p->v_stride[i];
    a->os[i] = p->o_stride[i];
  }
  a->q_lens = p->q_lens;
  a->kv_lens = p->kv_lens;
  a->alibi = p->alibi_slopes;
  a->sm_scale = p->sm_scale;
  a->softcap = p->logits_soft_cap > 0.f ? p->logits_soft_cap : 0.f;
  a->causal = p->causal ? 1 : 0;
  a->window = p->sliding_window < 0 ? -1 : p->sliding_window;
  a->lse = p->lse;
  a->kv_offset = p->kv_offset;
  a->kv_total = p->kv_total;
  a->err = nullptr;
  a->num_sms = 148;
  a->xs_n = a->xs_slice = a->xs_row_base = 0;
  for (int i = 0; i < LLMX_SCATTER_MAX_DST; ++i) {
    a->xs_o[i] = nullptr;
    a->xs_lse[i] = nullptr;
  }
  return LLMX_OK;
}

llmx_status choose(const AttnArgs &a, int requested, int *algo) {
  if (requested == LLMX_ALGO_AUTO) {
    if (a.dtype == LLMX_FP32) {
      *algo = LLMX_ALGO_SIMT;
    } else if (decode_supports(a)) {
      *algo = LLMX_ALGO_DECODE;
    } else if (sm100_supports(a)) {
      *algo = LLMX_ALGO_TCGEN05;
    } else {
      *algo = LLMX_ALGO_SIMT;
    }
    return LLMX_OK;
  }
  if (requested == LLMX_ALGO_DECODE && !decode_supports(a))
    return fail(LLMX_ERR_UNSUPPORTED,
                "decode kernel needs fp16/bf16, max_q_len == 1, head_dim 64/128/256 and 16-byte "
                "aligned rows");
  if (requested == LLMX_ALGO_TCGEN05 && !sm100_supports(a))
    return fail(LLMX_ERR_UNSUPPORTED,
                "tcgen05 kernel needs fp16/bf16, head_dim 64, 128 or 256, sm_scale > 0 and 16-byte aligned rows");
  *algo = requested;
  return LLMX_OK;
}

llmx_status current_device(int *dev, const DeviceInfo **info) {
  if (cudaGetDevice(dev) != cudaSuccess) return fail(LLMX_ERR_NO_DEVICE, "no CUDA device");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(LLMX_ERR_NO_DEVICE, "device index out of range");
  *info = &device_info(*dev);
  if (!(*info)->ok) return fail(LLMX_ERR_UNSUPPORTED, (*info)->why);
  return LLMX_OK;
}

}  // namespace

llmx_status prepare_decode_request(const llmx_attn_params *p, AttnArgs *a) {
  llmx_status s = validate(p, a);
  if (s != LLMX_OK) return s;
  if (!decode_supports(*a))
    return fail(LLMX_ERR_UNSUPPORTED,
                "decode kernel needs fp16/bf16, max_q_len == 1, head_dim 64/128/256 and 16-byte "
                "aligned rows");
  int dev = 0;
  const DeviceInfo *info = nullptr;
  s = current_device(&dev, &info);
  if (s != LLMX_OK) return s;
  a->err = info->err;
  a->num_sms = info->num_sms;
  return LLMX_OK;
}

llmx_status record_error(llmx_status s, const char *msg) { return fail(s, msg); }

}  // namespace llmx_b200

using namespace llmx_b200;

extern "C" {

llmx_status llmx_attn_params_init(llmx_attn_params *p) {
  if (p == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "params is NULL");
  std::memset(p, 0, sizeof(*p));
  p->causal = 1;
  p->sliding_window = -1;
  p->algo = LLMX_ALGO_AUTO;
  return LLMX_OK;
}

llmx_status llmx_attn_set_contiguous_strides(llmx_attn_params *p) {
  if (p == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "params is NULL");
  const int64_t D = p->head_dim;
  p->q_stride[2] = p->o_stride[2] = D;
  p->q_stride[1] = p->o_stride[1] = D * p->n_heads;
  p->q_stride[0] = p->o_stride[0] = D * p->n_heads * p->max_q_len;
  p->k_stride[2] = p->v_stride[2] = D;
  p->k_stride[1] = p->v_stride[1] = D * p->n_kv_heads;
  p->k_stride[0] = p->v_stride[0] = D * p->n_kv_heads * p->max_kv_len;
  return LLMX_OK;
}

llmx_status llmx_attn_select_algo(const llmx_attn_params *p, int32_t *algo) {
  AttnArgs a;
  llmx_status s = validate(p, &a);
  if (s != LLMX_OK) return s;
  if (algo == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "algo is NULL");
  int chosen = 0;
  s = choose(a, p->algo, &chosen);
  if (s == LLMX_OK) *algo = chosen;
  return s;
}

llmx_status llmx_attn_workspace_size(const llmx_attn_params *p, size_t *bytes) {
  AttnArgs a;
  llmx_status s = validate(p, &a);
  if (s != LLMX_OK) return s;
  if (bytes == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "bytes is NULL");
  int algo = 0;
  s = choose(a, p->algo, &algo);
  if (s != LLMX_OK) return s;
  *bytes = 0;
  if (algo == LLMX_ALGO_DECODE) {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
      const DeviceInfo &info = device_info(dev);
      if (info.ok) a.num_sms = info.num_sms;
    }
    *bytes = plan_decode(a, SIZE_MAX, true).ws_bytes;
  } else if (algo == LLMX_ALGO_TCGEN05) {
    *bytes = kSm100WorkspaceBytes;
  }
  return LLMX_OK;
}

llmx_status llmx_attn_fwd(const llmx_attn_params *p, void *stream) {
  AttnArgs a;
  llmx_status s = validate(p, &a);
  if (s != LLMX_OK) return s;
  int algo = 0;
  s = choose(a, p->algo, &algo);
  if (s != LLMX_OK) return s;
  int dev = 0;
  const DeviceInfo *info = nullptr;
  s = current_device(&dev, &info);
  if (s != LLMX_OK) return s;
  a.err = info->err;
  a.num_sms = info->num_sms;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  switch (algo) {
    case LLMX_ALGO_SIMT: e = launch_simt(a, st); break;
    case LLMX_ALGO_DECODE: {
      DecodePlan plan = plan_decode(a, p->workspace_bytes, p->workspace != nullptr);
      if (plan.n_splits > 1 && !aligned16(p->workspace))
        return fail(LLMX_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
      e = launch_decode(a, plan, p->workspace, st);
      break;
    }
    case LLMX_ALGO_TCGEN05: e = launch_sm100(a, p->workspace, p->workspace_bytes, st); break;
  }
  if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("launch failed: ") + cudaGetErrorString(e));
  return LLMX_OK;
}

llmx_status llmx_attn_fwd_scatter(const llmx_attn_params *p, const llmx_row_scatter *x, void *stream) {
  AttnArgs a;
  llmx_status s = validate(p, &a);
  if (s != LLMX_OK) return s;
  if (x == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "scatter: x is NULL");
  int algo = 0;
  s = choose(a, p->algo, &algo);
  if (s != LLMX_OK) return s;
  if (algo != LLMX_ALGO_TCGEN05 || a.D == 256)
    return fail(LLMX_ERR_UNSUPPORTED, "scatter: needs the tensor-core prefill (fp16/bf16, head_dim 64 or 128)");
  if (x->n_dst < 1 || x->n_dst > LLMX_SCATTER_MAX_DST)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "scatter: n_dst must be in [1, 8]");
  if (x->slice_rows < 16 || x->slice_rows % 16 || x->row_base < 0 || x->row_base % 16)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "scatter: slice_rows and row_base must be multiples of 16");
  const long long last = (long long)x->row_base + a.Sq - 1;
  if (last / x->slice_rows >= x->n_dst)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "scatter: rows past the last destination's slice");
  for (int d = x->row_base / x->slice_rows; d <= (int)(last / x->slice_rows); ++d)
    if (!aligned16(x->o[d]) || x->o[d] == nullptr || x->lse[d] == nullptr)
      return fail(LLMX_ERR_INVALID_ARGUMENT, "scatter: every destination that gets rows needs o (16-byte aligned) and lse");
  a.xs_n = x->n_dst;
  a.xs_slice = x->slice_rows;
  a.xs_row_base = x->row_base;
  for (int d = 0; d < LLMX_SCATTER_MAX_DST; ++d) {
    a.xs_o[d] = d < x->n_dst ? x->o[d] : nullptr;
    a.xs_lse[d] = d < x->n_dst ? x->lse[d] : nullptr;
  }
  int dev = 0;
  const DeviceInfo *info = nullptr;
  s = current_device(&dev, &info);
  if (s != LLMX_OK) return s;
  a.err = info->err;
  a.num_sms = info->num_sms;
  const cudaError_t e = launch_sm100(a, p->workspace, p->workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("launch failed: ") + cudaGetErrorString(e));
  return LLMX_OK;
}

llmx_status llmx_ipc_alloc(size_t bytes, void **ptr, void *handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0)
    return fail(LLMX_ERR_INVALID_ARGUMENT, "ipc alloc: ptr, handle and a size are required");
  static_assert(sizeof(cudaIpcMemHandle_t) == LLMX_IPC_HANDLE_BYTES, "IPC handle size");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    return fail(LLMX_ERR_CUDA, std::string("ipc alloc: ") + cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return LLMX_OK;
}

llmx_status llmx_ipc_open(const void *handle, void **ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(LLMX_ERR_INVALID_ARGUMENT, "ipc open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("ipc open: ") + cudaGetErrorString(e));
  return LLMX_OK;
}

llmx_status llmx_ipc_close(void *ptr) {
  if (ptr == nullptr) return LLMX_OK;  // nothing was opened
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("ipc close: ") + cudaGetErrorString(e));
  return LLMX_OK;
}

llmx_status llmx_ipc_free(void *ptr) {
  if (ptr == nullptr) return LLMX_OK;  // as free(NULL)
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("ipc free: ") + cudaGetErrorString(e));
  return LLMX_OK;
}

llmx_status llmx_single_mha_attention_c(void *output, const void *q, const void *k, const void *v,
                                        const float *alibi_slopes, int32_t dtype, int32_t q_len,
                                        int32_t kv_len, int32_t n_heads, int32_t n_kv_heads,
                                        int32_t head_dim, float sm_scale, int32_t sliding_window,
                                        float logits_soft_cap, void *stream) {
  llmx_attn_params p;
  llmx_attn_params_init(&p);
  p.dtype = dtype;
  p.batch = 1;
  p.n_heads = n_heads;
  p.n_kv_heads = n_kv_heads;
  p.head_dim = head_dim;
  p.max_q_len = q_len;
  p.max_kv_len = kv_len;
  p.q = q;
  p.k = k;
  p.v = v;
  p.o = output;
  p.alibi_slopes = alibi_slopes;
  p.sm_scale = sm_scale;
  p.causal = 1;
  p.sliding_window = sliding_window;
  p.logits_soft_cap = logits_soft_cap;
  llmx_attn_set_contiguous_strides(&p);
  return llmx_attn_fwd(&p, stream);
}

llmx_status llmx_attn_device_status(int32_t device, int32_t clear) {
  if (device < 0 || device >= kMaxDevices) return fail(LLMX_ERR_INVALID_ARGUMENT, "bad device");
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(LLMX_ERR_NO_DEVICE, "no CUDA device");
  if (prev != device && cudaSetDevice(device) != cudaSuccess)
    return fail(LLMX_ERR_NO_DEVICE, "cudaSetDevice failed");
  unsigned int word = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&word, g_device_error_word, sizeof(word));
  if (e == cudaSuccess && clear && word) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error_word, &zero, sizeof(zero));
  }
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, cudaGetErrorString(e));
  if (word & kDevErrTimeout) return fail(LLMX_ERR_TIMEOUT, "a device-side bounded wait expired");
  if (word & kDevErrTmemAlloc) return fail(LLMX_ERR_TIMEOUT, "tensor-memory allocation timed out");
  return LLMX_OK;
}

const char *llmx_status_string(llmx_status s) {
  switch (s) {
    case LLMX_OK: return "ok";
    case LLMX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LLMX_ERR_UNSUPPORTED: return "unsupported";
    case LLMX_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case LLMX_ERR_CUDA: return "CUDA error";
    case LLMX_ERR_TIMEOUT: return "device wait timed out";
    case LLMX_ERR_NO_DEVICE: return "no device";
  }
  return "unknown status";
}

const char *llmx_attn_last_error(void) { return g_last_error.c_str(); }

int32_t llmx_attn_abi_version(void) { return LLMX_ATTN_ABI_VERSION; }

}  // extern "C"
