// llmx::Tensor -- the tensor type llmx's attention op takes.
//
// Same public surface as the reference (include/llmx/tensor.h:17-177):
// ScalarType, DeviceType, Device and the cpu0 / cuda0..cuda7 shorthands,
// MemInfo, DataPtr, Tensor with dims/strides/capacity, allocate / resize /
// to_device, and the llmx_allocate / llmx_free / llmx_mem_info / llmx_copy
// helpers, so code written against the reference header compiles unchanged.
// Differences, all internal:
//  * CUDA tensors live in device memory (cudaMalloc + zero fill) instead of
//    managed memory (tensor.cpp:64-70);
//  * ownership is a shared control block, so copies share storage and the
//    last owner frees it (the reference keeps a refcount map, tensor.cpp:155-160);
//  * a Tensor built on an external pointer never owns it (tensor.cpp:218-224).
#pragma once

#include <cstddef>
#include <functional>
#include <memory>
#include <numeric>
#include <optional>
#include <vector>

namespace llmx {

enum class ScalarType { kFP32, kFP16, kBF16 };

size_t get_scalar_size(ScalarType dtype);

enum class DeviceType { kCPU, kCUDA };

struct Device {
  DeviceType type = DeviceType::kCPU;
  int id = -1;

  Device() = default;
  Device(DeviceType type, int id = -1) : type(type), id(id) {}

  bool operator==(const Device &other) const { return type == other.type && id == other.id; }
  bool operator!=(const Device &other) const { return !(*this == other); }
};

// Device shorthands of the reference header (tensor.h:38-46).
#define cpu0 Device(DeviceType::kCPU)
#define cuda0 Device(DeviceType::kCUDA, 0)
#define cuda1 Device(DeviceType::kCUDA, 1)
#define cuda2 Device(DeviceType::kCUDA, 2)
#define cuda3 Device(DeviceType::kCUDA, 3)
#define cuda4 Device(DeviceType::kCUDA, 4)
#define cuda5 Device(DeviceType::kCUDA, 5)
#define cuda6 Device(DeviceType::kCUDA, 6)
#define cuda7 Device(DeviceType::kCUDA, 7)

// What llmx_allocate recorded about a block it returned (tensor.h:48-52).
struct MemInfo {
  void *data;
  std::size_t nbytes;
  Device device;
};

// Zero-filled storage on `device` (64-byte aligned host memory, or CUDA
// device memory), recorded so that llmx_free / llmx_mem_info find it.  The
// record is process-wide and guarded by a mutex (the reference keeps one
// unguarded map per translation unit, tensor.h:54-67).
void *llmx_allocate(size_t nbytes, Device device);
// Frees a block llmx_allocate returned; pointers it did not return are
// ignored, as in the reference (tensor.cpp:134-146).
void llmx_free(void *data);
// Frees `data` as memory of `device` (also accepted for blocks the library
// did not allocate: host memory from malloc, device memory from cudaMalloc).
void llmx_free(void *data, Device device);
// The record of a block llmx_allocate returned, or nullopt (tensor.cpp:148-153).
std::optional<MemInfo> llmx_mem_info(void *data);

// Stream-ordered pooling of CUDA storage (off by default; also switched on by
// the environment variable LLMX_TENSOR_POOL=1 at the first CUDA allocation).
// When on, llmx_allocate takes CUDA blocks from the device's memory pool
// with cudaMallocAsync on the legacy default stream (zero-filled there) and
// llmx_free returns them with cudaFreeAsync on the same stream, keeping the
// pool's memory cached, so repeated tensor allocation costs no cudaMalloc /
// cudaFree and no device-wide synchronisation.  The reference runs all of
// its work on the legacy stream (attention_api.cpp:55), which orders these
// frees after it.  A caller that uses a tensor on a non-blocking stream must
// synchronise that stream before the tensor's storage is freed, or the pool
// may hand the block to another tensor while the work still runs; with the
// pool off, cudaFree's implicit synchronisation covers that case.  Blocks
// keep the mode they were allocated in.
void llmx_set_cuda_pool(bool enabled);
bool llmx_cuda_pool_enabled();
void llmx_copy(Device src_device, Device dst_device, const void *src, void *dst, size_t nbytes);
// Element-type conversion of `num` contiguous elements in device-addressable
// memory (src/tensor.cpp:108-118), on the legacy stream like the reference's
// scalar_convert_kernel launch.  Same types copy.  Throws std::runtime_error
// on a failing or refused launch (pageable host pointers are refused).
void llmx_copy(ScalarType src_dtype, ScalarType dst_dtype, const void *src, void *dst, size_t num);

// Pointer plus (for storage the allocator made) a shared owner.
class DataPtr {
 public:
  DataPtr() = default;
  DataPtr(void *ptr) : ptr_(ptr) {}  // non-owning
  DataPtr(void *ptr, Device device);          // owning: frees with llmx_free

  void *ptr() const noexcept { return ptr_; }
  template <typename T>
  T *ptr() const noexcept {
    return reinterpret_cast<T *>(ptr_);
  }
  bool owns() const noexcept { return owner_ != nullptr; }
  long use_count() const noexcept { return owner_ ? owner_.use_count() : 0; }
  bool operator==(std::nullptr_t) const noexcept { return ptr_ == nullptr; }
  bool operator!=(std::nullptr_t) const noexcept { return ptr_ != nullptr; }

 private:
  void *ptr_ = nullptr;
  std::shared_ptr<void> owner_;
};

class Tensor {
 public:
  Tensor() = default;
  Tensor(const std::vector<int> &dims, ScalarType dtype, Device device);  // metadata; allocate() adds storage
  Tensor(void *data, const std::vector<int> &dims, ScalarType dtype, Device device);  // wraps

  ScalarType dtype() const noexcept { return dtype_; }
  void dtype(ScalarType dtype) noexcept { dtype_ = dtype; }
  std::vector<int> dims() const noexcept { return dims_; }
  int dim(int axis) const noexcept { return dims_[axis]; }
  int stride(int axis) const noexcept { return strides_[axis]; }
  int ndim() const noexcept { return static_cast<int>(dims_.size()); }
  Device device() const noexcept { return device_; }
  const DataPtr &data() const noexcept { return data_; }
  DataPtr &data() noexcept { return data_; }
  const void *const_data_ptr() const noexcept { return data_.ptr(); }
  void *data_ptr() noexcept { return data_.ptr(); }
  template <typename T>
  const T *const_data_ptr() const noexcept {
    return data_.template ptr<T>();
  }
  template <typename T>
  T *data_ptr() noexcept {
    return data_.template ptr<T>();
  }

  bool is_valid() const noexcept { return data_.ptr() != nullptr && capacity_ > 0; }
  bool contiguous() const noexcept;
  // Bytes of storage held.  Tracked in bytes, so a tensor whose dtype was
  // changed to a wider type reallocates on allocate() even at equal numel.
  size_t nbytes() const noexcept { return storage_bytes_; }
  size_t capacity() const noexcept { return capacity_; }
  size_t count(int axis = 0) const noexcept { return size_t(dims_[axis]) * strides_[axis]; }
  size_t numel() const noexcept {
    return std::accumulate(dims_.begin(), dims_.end(), size_t(1), std::multiplies<>{});
  }

  // Makes room for numel() elements (reallocating, zeroed, only when growing).
  void allocate();
  // Metadata-only reshape; storage is kept (tensor_test.cpp:62-100).
  void resize(const std::vector<int> &dims);
  // Moves storage to `device`, copying the contents when `transfer`.
  void to_device(Device device, bool transfer = true);

 private:
  void set_dims(const std::vector<int> &dims);

  DataPtr data_;
  ScalarType dtype_ = ScalarType::kFP32;
  std::vector<int> dims_;
  std::vector<int> strides_;
  size_t capacity_ = 0;
  size_t storage_bytes_ = 0;
  Device device_ = Device(DeviceType::kCPU);
};

}  // namespace llmx
