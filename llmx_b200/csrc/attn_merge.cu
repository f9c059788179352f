// Log-sum-exp merge of attention partials over disjoint key sets (KV split).
//
// A query row's attention over keys K = K_1 u ... u K_n is recovered exactly
// from the partial results (O_c, lse_c) over each K_c:
//   lse = log sum_c exp(lse_c),   O = sum_c exp(lse_c - lse) O_c.
// The split-KV decode combine does this for splits inside one launch
// (attn_decode.cu); these two kernels do it for partials held in separate
// tensors, around a cross-GPU sum:
//   scale:  num[b,s,h,:] = sum_c w_c O_c[b,s,h,:],  wsum[b,h,s] = sum_c w_c,
//           w_c = exp(lse_c - m)  (m: the row max over every shard, 0 terms
//           for partials that saw no key);
//   finish: O = num / wsum (0 where wsum == 0), lse = m + log(wsum).
// Between them the caller all-reduces [num | wsum] (SUM) over the ranks.
// Same running max / sum algebra as the reference's online softmax
// (softmax.h:53-110), applied across shards instead of key blocks.
//
// Bandwidth-bound elementwise kernels.  A block takes one (b, h) and a run of
// rows_of(D) consecutive s: the per-row weights come from contiguous lse /
// row-max entries ([B, H, S] layout) into shared memory once, then every
// thread moves four 16-byte units of the rows' D elements (units of one row
// are adjacent lanes, so each row's D contiguous elements are read in one
// pass); all loads of a thread are issued before its arithmetic.  Every byte
// is read or written once.
#include "common.cuh"

namespace llmx_b200 {
namespace {

constexpr int kMaxParts = 8;
constexpr int kMergeThreads = 256;
constexpr int kUnitsPerThread = 4;
constexpr int kMaxRows = 128;

struct MergeArgs {
  int n_parts, B, S, H, D, dtype;
  const void *o[kMaxParts];       // [B, S, H, D] contiguous, input dtype
  const float *lse[kMaxParts];    // [B, H, S]
  const float *m;                 // [B, H, S] row max over all shards
  float *num;                     // [B, S, H, D] fp32
  float *wsum;                    // [B, H, S]
  void *out;                      // [B, S, H, D] input dtype
  float *lse_out;                 // [B, H, S] or null
};

// Rows per block: enough for kUnitsPerThread 8-element units per thread.
__host__ __device__ inline int rows_of(int D) {
  const int r = kMergeThreads * kUnitsPerThread / (D / 8);
  return r < 1 ? 1 : (r > kMaxRows ? kMaxRows : r);
}

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) merge_scale_kernel(MergeArgs a) {
  __shared__ float w_s[kMaxParts][kMaxRows];
  const int R = rows_of(a.D), V = a.D / 8;
  const int h = blockIdx.y, b = blockIdx.z;
  const int s0 = blockIdx.x * R;
  const long long lrow = ((long long)b * a.H + h) * a.S;  // [B, H, S] row base
  for (int r = threadIdx.x; r < R; r += kMergeThreads) {
    const int s = s0 + r;
    if (s >= a.S) break;
    const float m = a.m[lrow + s];
    const float m_safe = isinf(m) ? 0.f : m;
    float ws = 0.f;
    for (int c = 0; c < a.n_parts; ++c) {
      const float l = a.lse[c][lrow + s];
      const float w = (l == -CUDART_INF_F) ? 0.f : expf(l - m_safe);
      w_s[c][r] = w;
      ws += w;
    }
    a.wsum[lrow + s] = ws;
  }
  __syncthreads();
  const int rows = min(R, a.S - s0);
  const int n_units = rows * V;
  // Per partial: the thread's four units loaded first, then accumulated.
  float acc[kUnitsPerThread][8];
#pragma unroll
  for (int k = 0; k < kUnitsPerThread; ++k)
#pragma unroll
    for (int x = 0; x < 8; ++x) acc[k][x] = 0.f;
  for (int c = 0; c < a.n_parts; ++c) {
    const T *src = static_cast<const T *>(a.o[c]);
    uint4 raw[kUnitsPerThread];
#pragma unroll
    for (int k = 0; k < kUnitsPerThread; ++k) {
      const int idx = threadIdx.x + k * kMergeThreads;
      raw[k] = make_uint4(0u, 0u, 0u, 0u);
      if (idx < n_units) {
        const int r = idx / V, u = idx - r * V;
        if (w_s[c][r] != 0.f)
          raw[k] = *reinterpret_cast<const uint4 *>(src + (((long long)b * a.S + s0 + r) * a.H + h) * a.D + u * 8);
      }
    }
#pragma unroll
    for (int k = 0; k < kUnitsPerThread; ++k) {
      const int idx = threadIdx.x + k * kMergeThreads;
      if (idx < n_units) {
        const float w = w_s[c][idx / V];
        float f[8];
        unpack8<T>(raw[k], f);
#pragma unroll
        for (int x = 0; x < 8; ++x) acc[k][x] = fmaf(w, f[x], acc[k][x]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kUnitsPerThread; ++k) {
    const int idx = threadIdx.x + k * kMergeThreads;
    if (idx >= n_units) break;
    const int r = idx / V, u = idx - r * V;
    float4 *dst = reinterpret_cast<float4 *>(a.num + (((long long)b * a.S + s0 + r) * a.H + h) * a.D + u * 8);
    dst[0] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
    dst[1] = make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) merge_finish_kernel(MergeArgs a) {
  __shared__ float inv_s[kMaxRows];
  const int R = rows_of(a.D), V = a.D / 8;
  const int h = blockIdx.y, b = blockIdx.z;
  const int s0 = blockIdx.x * R;
  const long long lrow = ((long long)b * a.H + h) * a.S;
  for (int r = threadIdx.x; r < R; r += kMergeThreads) {
    const int s = s0 + r;
    if (s >= a.S) break;
    const float ws = a.wsum[lrow + s];
    inv_s[r] = ws > 0.f ? 1.f / ws : 0.f;
    if (a.lse_out != nullptr) {
      const float m = a.m[lrow + s];
      a.lse_out[lrow + s] = ws > 0.f ? (isinf(m) ? 0.f : m) + logf(ws) : -CUDART_INF_F;
    }
  }
  __syncthreads();
  const int rows = min(R, a.S - s0);
  const int n_units = rows * V;
  float4 x[kUnitsPerThread][2];
#pragma unroll
  for (int k = 0; k < kUnitsPerThread; ++k) {
    const int idx = threadIdx.x + k * kMergeThreads;
    if (idx >= n_units) break;
    const int r = idx / V, u = idx - r * V;
    const long long e = (((long long)b * a.S + s0 + r) * a.H + h) * a.D + u * 8;
    const float4 *src = reinterpret_cast<const float4 *>(a.num + e);
    x[k][0] = src[0];
    x[k][1] = src[1];
  }
#pragma unroll
  for (int k = 0; k < kUnitsPerThread; ++k) {
    const int idx = threadIdx.x + k * kMergeThreads;
    if (idx >= n_units) break;
    const int r = idx / V, u = idx - r * V;
    const long long e = (((long long)b * a.S + s0 + r) * a.H + h) * a.D + u * 8;
    const float inv = inv_s[r];
    const float f[8] = {x[k][0].x * inv, x[k][0].y * inv, x[k][0].z * inv, x[k][0].w * inv,
                        x[k][1].x * inv, x[k][1].y * inv, x[k][1].z * inv, x[k][1].w * inv};
    *reinterpret_cast<uint4 *>(static_cast<T *>(a.out) + e) = pack8<T>(f);
  }
}

dim3 merge_grid(const MergeArgs &a) {
  const int R = rows_of(a.D);
  return dim3((unsigned)((a.S + R - 1) / R), (unsigned)a.H, (unsigned)a.B);
}

cudaError_t launch_scale(const MergeArgs &a, cudaStream_t st) {
  if (a.dtype == LLMX_FP16)
    merge_scale_kernel<__half><<<merge_grid(a), kMergeThreads, 0, st>>>(a);
  else
    merge_scale_kernel<__nv_bfloat16><<<merge_grid(a), kMergeThreads, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_finish(const MergeArgs &a, cudaStream_t st) {
  if (a.dtype == LLMX_FP16)
    merge_finish_kernel<__half><<<merge_grid(a), kMergeThreads, 0, st>>>(a);
  else
    merge_finish_kernel<__nv_bfloat16><<<merge_grid(a), kMergeThreads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace
}  // namespace llmx_b200

using namespace llmx_b200;

static llmx_status merge_common(MergeArgs *m, int32_t n_parts, const void *const *outs, const float *const *lses,
                                int32_t dtype, int32_t B, int32_t S, int32_t H, int32_t D) {
  if (n_parts < 0 || n_parts > kMaxParts)
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: n_parts must be in [0, 8]");
  if (dtype != LLMX_FP16 && dtype != LLMX_BF16)
    return record_error(LLMX_ERR_UNSUPPORTED, "lse merge: dtype must be fp16 or bf16");
  if (B < 1 || S < 1 || H < 1 || D < 8 || D % 8)
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: B, S, H >= 1 and head_dim a multiple of 8");
  if (B > 65535 || H > 65535 || D > 8192)
    return record_error(LLMX_ERR_INVALID_ARGUMENT,
                        "lse merge: batch and n_heads must be at most 65535, head_dim at most 8192");
  m->n_parts = n_parts;
  m->B = B;
  m->S = S;
  m->H = H;
  m->D = D;
  m->dtype = dtype;
  for (int c = 0; c < n_parts; ++c) {
    if (outs == nullptr || lses == nullptr || outs[c] == nullptr || lses[c] == nullptr ||
        (reinterpret_cast<uintptr_t>(outs[c]) & 15u))
      return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: partial pointers must be non-NULL, 16-byte aligned");
    m->o[c] = outs[c];
    m->lse[c] = lses[c];
  }
  return LLMX_OK;
}

extern "C" llmx_status llmx_attn_lse_merge_scale(int32_t n_parts, const void *const *outs, const float *const *lses,
                                                 const float *row_max, int32_t dtype, int32_t batch, int32_t seq,
                                                 int32_t n_heads, int32_t head_dim, float *num, float *wsum,
                                                 void *stream) {
  MergeArgs m{};
  llmx_status s = merge_common(&m, n_parts, outs, lses, dtype, batch, seq, n_heads, head_dim);
  if (s != LLMX_OK) return s;
  if (row_max == nullptr || num == nullptr || wsum == nullptr || (reinterpret_cast<uintptr_t>(num) & 15u))
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: row_max, num, wsum required (num 16-byte aligned)");
  m.m = row_max;
  m.num = num;
  m.wsum = wsum;
  cudaError_t e = launch_scale(m, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LLMX_OK : record_error(LLMX_ERR_CUDA, cudaGetErrorString(e));
}

extern "C" llmx_status llmx_attn_lse_merge_finish(const float *num, const float *wsum, const float *row_max,
                                                  int32_t dtype, int32_t batch, int32_t seq, int32_t n_heads,
                                                  int32_t head_dim, void *out, float *lse_out, void *stream) {
  MergeArgs m{};
  llmx_status s = merge_common(&m, 0, nullptr, nullptr, dtype, batch, seq, n_heads, head_dim);
  if (s != LLMX_OK) return s;
  if (num == nullptr || wsum == nullptr || row_max == nullptr || out == nullptr ||
      (reinterpret_cast<uintptr_t>(num) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u))
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: num, wsum, row_max, out required and aligned");
  m.num = const_cast<float *>(num);
  m.wsum = const_cast<float *>(wsum);
  m.m = row_max;
  m.out = out;
  m.lse_out = lse_out;
  cudaError_t e = launch_finish(m, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LLMX_OK : record_error(LLMX_ERR_CUDA, cudaGetErrorString(e));
}
