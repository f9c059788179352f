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
// Bandwidth-bound elementwise kernels: one warp per (b, s, h) row, 16-byte
// vector accesses, every byte read or written once.
#include "common.cuh"

namespace llmx_b200 {
namespace {

constexpr int kMaxParts = 8;

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

template <typename T>
__global__ void __launch_bounds__(256) merge_scale_kernel(MergeArgs a) {
  const long long row = (long long)blockIdx.x * 8 + threadIdx.x / 32;  // (b, s, h)
  const int lane = threadIdx.x % 32;
  const long long rows = (long long)a.B * a.S * a.H;
  if (row >= rows) return;
  const int h = (int)(row % a.H);
  const long long bs = row / a.H;
  const int s = (int)(bs % a.S), b = (int)(bs / a.S);
  const long long li = ((long long)b * a.H + h) * a.S + s;
  const float m = a.m[li];
  const float m_safe = isinf(m) ? 0.f : m;
  float w[kMaxParts];
  float ws = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxParts; ++c) {
    w[c] = 0.f;
    if (c < a.n_parts) {
      const float l = a.lse[c][li];
      w[c] = (l == -CUDART_INF_F) ? 0.f : expf(l - m_safe);
      ws += w[c];
    }
  }
  // D / 8 lanes of 8 elements each
  for (int d0 = lane * 8; d0 < a.D; d0 += 32 * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < kMaxParts; ++c) {
      if (c < a.n_parts && w[c] != 0.f) {
        const T *src = static_cast<const T *>(a.o[c]) + row * a.D + d0;
        float f[8];
        unpack8<T>(*reinterpret_cast<const uint4 *>(src), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(w[c], f[e], acc[e]);
      }
    }
    float4 *dst = reinterpret_cast<float4 *>(a.num + row * a.D + d0);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  if (lane == 0) a.wsum[li] = ws;
}

template <typename T>
__global__ void __launch_bounds__(256) merge_finish_kernel(MergeArgs a) {
  const long long row = (long long)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const long long rows = (long long)a.B * a.S * a.H;
  if (row >= rows) return;
  const int h = (int)(row % a.H);
  const long long bs = row / a.H;
  const int s = (int)(bs % a.S), b = (int)(bs / a.S);
  const long long li = ((long long)b * a.H + h) * a.S + s;
  const float ws = a.wsum[li];
  const float inv = ws > 0.f ? 1.f / ws : 0.f;
  for (int d0 = lane * 8; d0 < a.D; d0 += 32 * 8) {
    const float4 *src = reinterpret_cast<const float4 *>(a.num + row * a.D + d0);
    const float4 x = src[0], y = src[1];
    const float f[8] = {x.x * inv, x.y * inv, x.z * inv, x.w * inv, y.x * inv, y.y * inv, y.z * inv, y.w * inv};
    *reinterpret_cast<uint4 *>(static_cast<T *>(a.out) + row * a.D + d0) = pack8<T>(f);
  }
  if (lane == 0 && a.lse_out != nullptr) {
    const float m = a.m[li];
    a.lse_out[li] = ws > 0.f ? (isinf(m) ? 0.f : m) + logf(ws) : -CUDART_INF_F;
  }
}

cudaError_t launch_scale(const MergeArgs &a, cudaStream_t st) {
  const unsigned blocks = (unsigned)(((long long)a.B * a.S * a.H + 7) / 8);
  if (a.dtype == LLMX_FP16)
    merge_scale_kernel<__half><<<blocks, 256, 0, st>>>(a);
  else
    merge_scale_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_finish(const MergeArgs &a, cudaStream_t st) {
  const unsigned blocks = (unsigned)(((long long)a.B * a.S * a.H + 7) / 8);
  if (a.dtype == LLMX_FP16)
    merge_finish_kernel<__half><<<blocks, 256, 0, st>>>(a);
  else
    merge_finish_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(a);
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
