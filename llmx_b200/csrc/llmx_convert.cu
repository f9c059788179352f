// Element-type conversion between fp32, fp16 and bf16 (llmx's to_fp32 /
// to_fp16 / to_bf16 ops).
//
// Reference: scalar_convert_kernel (src/scalar.cu:33-46) converts one element
// per thread in 256-thread blocks with round-to-nearest casts
// (__float2half / __float2bfloat16; 16-bit to 16-bit through fp32,
// scalar.cu:6-31).  Same rounding here; the kernel is HBM-bound, so each
// thread moves 8 elements per step with 16-byte vector accesses (two for
// fp32) in a grid-stride loop over a grid of whole waves (8 resident blocks
// per SM).  A request whose source and destination types match is a plain
// copy (the reference's same-type converter writes nothing, scalar.h:13-15).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "attn_internal.h"
#include "common.cuh"

namespace llmx_b200 {
namespace {

template <typename S>
__device__ __forceinline__ void load8(const S *p, float (&f)[8]) {
  if constexpr (std::is_same<S, float>::value) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    unpack8<S>(*reinterpret_cast<const uint4 *>(p), f);
  }
}

template <typename Dt>
__device__ __forceinline__ void store8(Dt *p, const float (&f)[8]) {
  if constexpr (std::is_same<Dt, float>::value) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    *reinterpret_cast<uint4 *>(p) = pack8<Dt>(f);
  }
}

template <typename S, typename Dt>
__global__ void __launch_bounds__(256) convert_kernel(const S *__restrict__ src, Dt *__restrict__ dst, size_t n,
                                                      int vec_ok) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec_ok) {
    const size_t n8 = n / 8;
    for (size_t i = tid; i < n8; i += stride) {
      float f[8];
      load8<S>(src + i * 8, f);
      store8<Dt>(dst + i * 8, f);
    }
    for (size_t i = n8 * 8 + tid; i < n; i += stride) dst[i] = Elem<Dt>::from_f(Elem<S>::to_f(src[i]));
  } else {
    for (size_t i = tid; i < n; i += stride) dst[i] = Elem<Dt>::from_f(Elem<S>::to_f(src[i]));
  }
}

template <typename S, typename Dt>
cudaError_t launch(const void *src, void *dst, size_t n, int num_sms, cudaStream_t st) {
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0;
  const size_t work = (n + 7) / 8;
  const size_t blocks_needed = (work + 255) / 256;
  const size_t waves = (size_t)num_sms * 8;  // 8 resident 256-thread blocks per SM
  const unsigned grid = (unsigned)(blocks_needed < waves ? (blocks_needed ? blocks_needed : 1) : waves);
  convert_kernel<S, Dt><<<grid, 256, 0, st>>>(static_cast<const S *>(src), static_cast<Dt *>(dst), n, vec_ok);
  return cudaGetLastError();
}

template <typename S>
cudaError_t launch_to(int dst_dtype, const void *src, void *dst, size_t n, int num_sms, cudaStream_t st) {
  switch (dst_dtype) {
    case LLMX_FP32: return launch<S, float>(src, dst, n, num_sms, st);
    case LLMX_FP16: return launch<S, __half>(src, dst, n, num_sms, st);
    case LLMX_BF16: return launch<S, __nv_bfloat16>(src, dst, n, num_sms, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace
}  // namespace llmx_b200

using namespace llmx_b200;

// The kernel dereferences both pointers, so each must be memory this device
// can address: its own allocation, managed memory, or pinned host memory.
// Pageable host memory and another device's allocation are rejected here
// instead of faulting in the kernel.
static bool device_addressable(const void *p, int dev) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  switch (a.type) {
    case cudaMemoryTypeDevice: return a.device == dev;
    case cudaMemoryTypeManaged: return true;
    case cudaMemoryTypeHost: return a.devicePointer != nullptr;
    default: return false;
  }
}

extern "C" llmx_status llmx_convert(const void *src, int32_t src_dtype, void *dst, int32_t dst_dtype, size_t n,
                                    void *stream) {
  if (src_dtype < LLMX_FP32 || src_dtype > LLMX_BF16 || dst_dtype < LLMX_FP32 || dst_dtype > LLMX_BF16)
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "llmx_convert: unknown dtype");
  if (n == 0) return LLMX_OK;
  if (src == nullptr || dst == nullptr) return record_error(LLMX_ERR_INVALID_ARGUMENT, "llmx_convert: NULL pointer");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_error(LLMX_ERR_CUDA, cudaGetErrorString(e));
  if (!device_addressable(src, dev) || !device_addressable(dst, dev))
    return record_error(LLMX_ERR_INVALID_ARGUMENT,
                        "llmx_convert: src and dst must be memory of the current device (or managed / pinned)");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (src_dtype == dst_dtype) {
    const size_t es = src_dtype == LLMX_FP32 ? 4 : 2;
    e = cudaMemcpyAsync(dst, src, n * es, cudaMemcpyDefault, st);
  } else {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    switch (src_dtype) {
      case LLMX_FP32: e = launch_to<float>(dst_dtype, src, dst, n, sms, st); break;
      case LLMX_FP16: e = launch_to<__half>(dst_dtype, src, dst, n, sms, st); break;
      default: e = launch_to<__nv_bfloat16>(dst_dtype, src, dst, n, sms, st); break;
    }
  }
  return e == cudaSuccess ? LLMX_OK : record_error(LLMX_ERR_CUDA, cudaGetErrorString(e));
}
