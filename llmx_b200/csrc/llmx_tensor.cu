// llmx::Tensor storage and copies (host code).  Semantics of the reference's
// src/tensor.cpp:1-263 that callers observe are kept: allocation zero-fills,
// resize is metadata-only, allocate() reallocates only when growing, and
// to_device moves (optionally copies) storage between host and a CUDA device.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "llmx/tensor.h"
#include "llmx_attn.h"

namespace llmx {
namespace {
void cuda_ok(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Blocks llmx_allocate returned, for llmx_free(void *) and llmx_mem_info,
// and which of them came from the stream-ordered pool.
std::mutex g_blocks_mu;
std::unordered_map<void *, MemInfo> &blocks() {
  static auto *m = new std::unordered_map<void *, MemInfo>();  // outlives static destructors
  return *m;
}
std::unordered_map<void *, bool> &pooled() {
  static auto *m = new std::unordered_map<void *, bool>();
  return *m;
}

// -1: not decided yet (read LLMX_TENSOR_POOL at the first CUDA allocation).
std::atomic<int> g_pool_mode{-1};

bool pool_on() {
  int m = g_pool_mode.load();
  if (m < 0) {
    const char *env = std::getenv("LLMX_TENSOR_POOL");
    int want = (env != nullptr && env[0] == '1') ? 1 : 0;
    g_pool_mode.compare_exchange_strong(m, want);
    m = g_pool_mode.load();
  }
  return m == 1;
}

// Keeps the freed memory of the current device's default pool cached (the
// pool would otherwise return it to the driver at the next synchronisation).
void retain_pool_memory(int dev) {
  static std::once_flag once[64];
  if (dev < 0 || dev >= 64) return;
  std::call_once(once[dev], [dev] {
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
  });
}

void release(void *data, Device device, bool from_pool) {
  if (device.type == DeviceType::kCPU) {
    std::free(data);
  } else if (from_pool) {
    // Freed on the legacy stream of the device whose pool holds the block.
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device.id < 0 ? 0 : device.id);
    cudaFreeAsync(data, 0);
    cudaSetDevice(prev);
  } else {
    cudaFree(data);
  }
}
}  // namespace

size_t get_scalar_size(ScalarType dtype) {
  switch (dtype) {
    case ScalarType::kFP32: return 4;
    case ScalarType::kFP16: return 2;
    case ScalarType::kBF16: return 2;
  }
  throw std::invalid_argument("unsupported scalar type");
}

void *llmx_allocate(size_t nbytes, Device device) {
  if (nbytes == 0) return nullptr;
  void *p = nullptr;
  if (device.type == DeviceType::kCPU) {
    if (posix_memalign(&p, 64, nbytes) != 0) throw std::bad_alloc();
    std::memset(p, 0, nbytes);
  } else {
    int prev = 0;
    cuda_ok(cudaGetDevice(&prev), "cudaGetDevice");
    const int dev = device.id < 0 ? 0 : device.id;
    cuda_ok(cudaSetDevice(dev), "cudaSetDevice");
    const bool from_pool = pool_on();
    cudaError_t e;
    if (from_pool) {
      retain_pool_memory(dev);
      e = cudaMallocAsync(&p, nbytes, 0);
      if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, nbytes, 0);
    } else {
      e = cudaMalloc(&p, nbytes);
      if (e == cudaSuccess) e = cudaMemset(p, 0, nbytes);
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess && p != nullptr) {
      if (from_pool)
        cudaFreeAsync(p, 0);
      else
        cudaFree(p);
      p = nullptr;
    }
    cuda_ok(e, from_pool ? "cudaMallocAsync" : "cudaMalloc");
    std::lock_guard<std::mutex> lock(g_blocks_mu);
    if (from_pool) pooled()[p] = true;
  }
  std::lock_guard<std::mutex> lock(g_blocks_mu);
  blocks()[p] = MemInfo{p, nbytes, device};
  return p;
}

void llmx_set_cuda_pool(bool enabled) { g_pool_mode.store(enabled ? 1 : 0); }

bool llmx_cuda_pool_enabled() { return pool_on(); }

void llmx_free(void *data) {
  if (data == nullptr) return;
  Device device;
  bool from_pool = false;
  {
    std::lock_guard<std::mutex> lock(g_blocks_mu);
    auto it = blocks().find(data);
    if (it == blocks().end()) return;
    device = it->second.device;
    blocks().erase(it);
    from_pool = pooled().erase(data) > 0;
  }
  release(data, device, from_pool);
}

void llmx_free(void *data, Device device) {
  if (data == nullptr) return;
  bool from_pool = false;
  {
    std::lock_guard<std::mutex> lock(g_blocks_mu);
    blocks().erase(data);
    from_pool = pooled().erase(data) > 0;
  }
  release(data, device, from_pool);
}

std::optional<MemInfo> llmx_mem_info(void *data) {
  std::lock_guard<std::mutex> lock(g_blocks_mu);
  auto it = blocks().find(data);
  if (it == blocks().end()) return std::nullopt;
  return it->second;
}

void llmx_copy(Device src_device, Device dst_device, const void *src, void *dst,
                        size_t nbytes) {
  if (nbytes == 0) return;
  if (src == nullptr || dst == nullptr) throw std::invalid_argument("llmx_copy: null pointer");
  if (src_device.type == DeviceType::kCPU && dst_device.type == DeviceType::kCPU) {
    std::memcpy(dst, src, nbytes);
    return;
  }
  cuda_ok(cudaMemcpy(dst, src, nbytes, cudaMemcpyDefault), "cudaMemcpy");
}

void llmx_copy(ScalarType src_dtype, ScalarType dst_dtype, const void *src, void *dst, size_t num) {
  if (num == 0) return;
  if (src == nullptr || dst == nullptr) throw std::invalid_argument("llmx_copy: null pointer");
  const llmx_status s = llmx_convert(src, static_cast<int32_t>(src_dtype), dst, static_cast<int32_t>(dst_dtype), num,
                                     nullptr);
  if (s != LLMX_OK) throw std::runtime_error(std::string("llmx_copy: ") + llmx_attn_last_error());
}

DataPtr::DataPtr(void *ptr, Device device)
    : ptr_(ptr), owner_(ptr, [device](void *p) { llmx_free(p, device); }) {}

// Metadata only: storage comes with allocate(), as in the reference
// (tensor.cpp:213-217; tensor_test.cpp checks is_valid() is false here).
Tensor::Tensor(const std::vector<int> &dims, ScalarType dtype, Device device)
    : dtype_(dtype), device_(device) {
  set_dims(dims);
}

Tensor::Tensor(void *data, const std::vector<int> &dims, ScalarType dtype, Device device)
    : data_(data), dtype_(dtype), device_(device) {
  set_dims(dims);
  capacity_ = numel();
  storage_bytes_ = capacity_ * get_scalar_size(dtype_);
}

void Tensor::set_dims(const std::vector<int> &dims) {
  dims_ = dims;
  strides_.assign(dims.size(), 1);
  for (int i = static_cast<int>(dims.size()) - 2; i >= 0; --i) strides_[i] = strides_[i + 1] * dims[i + 1];
}

bool Tensor::contiguous() const noexcept {
  if (strides_.empty()) return true;
  if (strides_.back() != 1) return false;
  for (int i = static_cast<int>(dims_.size()) - 2; i >= 0; --i)
    if (strides_[i] != strides_[i + 1] * dims_[i + 1]) return false;
  return true;
}

void Tensor::allocate() {
  const size_t n = numel();
  const size_t need = n * get_scalar_size(dtype_);
  if (data_.ptr() != nullptr && need <= storage_bytes_) return;
  void *p = llmx_allocate(need, device_);
  data_ = DataPtr(p, device_);
  capacity_ = n;
  storage_bytes_ = need;
}

void Tensor::resize(const std::vector<int> &dims) { set_dims(dims); }

void Tensor::to_device(Device device, bool transfer) {
  if (device == device_) return;
  if (!is_valid()) {
    device_ = device;
    return;
  }
  void *p = llmx_allocate(storage_bytes_, device);
  if (transfer) llmx_copy(device_, device, data_.ptr(), p, storage_bytes_);
  data_ = DataPtr(p, device);
  device_ = device;
}

}  // namespace llmx
