// Device helpers shared by the attention kernels: element conversion,
// masking/score rules and the error word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

#include <type_traits>

#include "attn_internal.h"

namespace llmx_b200 {

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// 16 bytes (8 x 16-bit) -> 8 floats.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (sizeof(T) == 2 && std::is_same<T, __half>::value) {
      __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    } else {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162 *>(&w[i]);
      float2 p = __bfloat1622float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __half>::value) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t *>(&h);
    } else {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t *>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Streaming 16-byte load that skips L1 allocation (K/V are read once).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ int clamp_len(const int *lens, int b, int maxv) {
  if (lens == nullptr) return maxv;
  int x = lens[b];
  return x < 0 ? 0 : (x > maxv ? maxv : x);
}

// Score transform shared by every kernel: soft-cap then ALiBi.
// s = q.k * sm_scale;  cap > 0: s = tanh(s / cap) * cap  (params.h:35-50);
// s += slope * j                                          (mask.h:75-77).
__device__ __forceinline__ float score_transform(float dot, float sm_scale, float softcap,
                                                 float slope, int j) {
  float s = dot * sm_scale;
  if (softcap > 0.f) s = tanhf(s / softcap) * softcap;
  return s + slope * (float)j;
}

// Diagonal shift in local key indices: local key j is visible to query row i
// under the causal rule when j <= i + doff (mask.h:54-63), where
// doff = kfull - q_len - kv_offset and kfull is the full key length of the
// sequence (kv_total, or the local length when the keys are not sharded).
__device__ __forceinline__ int diag_shift(const AttnArgs &a, int ql, int kl) {
  const int kfull = a.kv_total > 0 ? a.kv_total : kl;
  return kfull - ql - a.kv_offset;
}

// Visibility of local key j to query row i, mask.h:41-81: inside the local
// length, on or below the (shifted) diagonal, inside the window.
__device__ __forceinline__ bool key_visible(int i, int j, int kl, int doff, int causal, int window) {
  if (j >= kl || j < 0) return false;
  const int diag = i + doff;
  if (causal && j > diag) return false;
  if (window >= 0 && (diag - j) > window) return false;
  return true;
}

__device__ __forceinline__ void raise_error(unsigned int *err, unsigned int code) {
  atomicOr(err, code);
}

}  // namespace llmx_b200
