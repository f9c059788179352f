// Log-sum-exp merge of attention partials over disjoint key sets (KV split).
//
// A query row's attention over keys K = K_1 u ... u K_n is recovered exactly
// from the partial results (O_c, lse_c) over each K_c:
//   m = max_c lse_c,  w_c = exp(lse_c - m),  W = sum_c w_c,
//   O = (sum_c w_c O_c) / W,  lse = m + log W.
// The split-KV decode combine does this for splits inside one launch
// (attn_decode.cu); this kernel does it for partials held in separate
// buffers: the local key chunks of one GPU, or the row slices that the
// KV-split exchange brought in from every GPU.  Each partial covers a range
// of output rows [row_lo, row_hi) (a GPU whose keys no row below row_lo can
// see under the causal mask computes and sends only rows >= row_lo); rows
// outside a partial's range get no term from it.  Same running max / sum
// algebra as the reference's online softmax (softmax.h:53-110), applied
// across shards instead of key blocks.
//
// Bandwidth-bound: a block takes one (b, h) and a run of rows_of(D)
// consecutive rows; the per-row weights go to shared memory once, then every
// thread moves four 16-byte units of the rows' D elements (units of one row
// are adjacent lanes); the first partial's loads are issued before the
// weights are computed.  A partial's O is read only inside its row range and used
// only where its weight is non-zero (rows its keys did not reach may hold
// anything).  Every byte is read or written once.
#include "common.cuh"

namespace llmx_b200 {
namespace {

constexpr int kMaxParts = 16;
constexpr int kMergeThreads = 256;
constexpr int kUnitsPerThread = 4;
constexpr int kMaxRows = 128;

struct PartDev {
  const void *o;
  const float *lse;
  long long os[3];  // batch, row, head (elements); rows counted from row_lo
  long long ls[2];  // batch, head (elements); rows unit-stride from row_lo
  int row_lo, row_hi;
};

struct MergeArgs {
  int n_parts, B, S, H, D;
  PartDev p[kMaxParts];
  void *out;
  long long outs[3];
  float *lse_out;  // [B, H, S] or null
};

// Rows per block: enough for kUnitsPerThread 8-element units per thread.
__host__ __device__ inline int rows_of(int D) {
  const int r = kMergeThreads * kUnitsPerThread / (D / 8);
  return r < 1 ? 1 : (r > kMaxRows ? kMaxRows : r);
}

template <typename T>
__global__ void __launch_bounds__(kMergeThreads, 4) lse_merge_kernel(const __grid_constant__ MergeArgs a) {
  __shared__ float w_s[kMaxParts][kMaxRows];
  __shared__ float inv_s[kMaxRows];
  const int R = rows_of(a.D), V = a.D / 8;
  // Heads are the fastest grid dimension: blocks running together read
  // whole rows (all heads) of the same row run, contiguous in memory.
  const int h = blockIdx.x, b = blockIdx.z;
  const int s0 = blockIdx.y * R;
  const int rows = min(R, a.S - s0);
  const int n_units = rows * V;
  // Partials in groups of kGroup (one: measured fastest on B200, with four
  // 256-thread blocks per SM; larger groups cost occupancy).  The first
  // group's O loads are issued before the weights are known (only rows
  // inside a part's range are read, so every load is in bounds), overlapping
  // the lse loads below; a loaded value is used only where its weight is
  // non-zero (rows a part's keys did not reach may hold anything).
  constexpr int kGroup = 1;
  uint4 raw[kGroup][kUnitsPerThread];
  auto load_group = [&](int c0) {
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const int c = c0 + g;
      const bool live = c < a.n_parts && !(s0 + rows <= a.p[c].row_lo || s0 >= a.p[c].row_hi);
      const T *src = live ? static_cast<const T *>(a.p[c].o) + b * a.p[c].os[0] + h * a.p[c].os[2] : nullptr;
#pragma unroll
      for (int k = 0; k < kUnitsPerThread; ++k) {
        const int idx = threadIdx.x + k * kMergeThreads;
        raw[g][k] = make_uint4(0u, 0u, 0u, 0u);
        if (live && idx < n_units) {
          const int r = idx / V, u = idx - r * V;
          const int s = s0 + r;
          if (s >= a.p[c].row_lo && s < a.p[c].row_hi)
            raw[g][k] = *reinterpret_cast<const uint4 *>(src + (long long)(s - a.p[c].row_lo) * a.p[c].os[1] + u * 8);
        }
      }
    }
  };
  load_group(0);
  for (int r = threadIdx.x; r < R; r += kMergeThreads) {
    const int s = s0 + r;
    if (s >= a.S) break;
    float l[kMaxParts];
#pragma unroll
    for (int c = 0; c < kMaxParts; ++c) {
      l[c] = -CUDART_INF_F;
      if (c < a.n_parts) {
        const PartDev &p = a.p[c];
        if (s >= p.row_lo && s < p.row_hi) l[c] = p.lse[b * p.ls[0] + h * p.ls[1] + (s - p.row_lo)];
      }
    }
    float m = -CUDART_INF_F;
#pragma unroll
    for (int c = 0; c < kMaxParts; ++c) m = fmaxf(m, l[c]);
    float ws = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxParts; ++c) {
      if (c < a.n_parts) {
        const float w = (l[c] == -CUDART_INF_F) ? 0.f : expf(l[c] - m);
        w_s[c][r] = w;
        ws += w;
      }
    }
    inv_s[r] = ws > 0.f ? 1.f / ws : 0.f;
    if (a.lse_out != nullptr)
      a.lse_out[((long long)b * a.H + h) * a.S + s] = ws > 0.f ? m + logf(ws) : -CUDART_INF_F;
  }
  __syncthreads();
  float acc[kUnitsPerThread][8];
#pragma unroll
  for (int k = 0; k < kUnitsPerThread; ++k)
#pragma unroll
    for (int x = 0; x < 8; ++x) acc[k][x] = 0.f;
  for (int c0 = 0; c0 < a.n_parts; c0 += kGroup) {
    if (c0 > 0) load_group(c0);
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const int c = c0 + g;
      if (c >= a.n_parts) break;
#pragma unroll
      for (int k = 0; k < kUnitsPerThread; ++k) {
        const int idx = threadIdx.x + k * kMergeThreads;
        if (idx < n_units) {
          const float w = w_s[c][idx / V];
          if (w != 0.f) {
            float f[8];
            unpack8<T>(raw[g][k], f);
#pragma unroll
            for (int x = 0; x < 8; ++x) acc[k][x] = fmaf(w, f[x], acc[k][x]);
          }
        }
      }
    }
  }
  T *dst = static_cast<T *>(a.out) + b * a.outs[0] + h * a.outs[2];
#pragma unroll
  for (int k = 0; k < kUnitsPerThread; ++k) {
    const int idx = threadIdx.x + k * kMergeThreads;
    if (idx >= n_units) break;
    const int r = idx / V, u = idx - r * V;
    const float inv = inv_s[r];
    float f[8];
#pragma unroll
    for (int x = 0; x < 8; ++x) f[x] = acc[k][x] * inv;
    *reinterpret_cast<uint4 *>(dst + (long long)(s0 + r) * a.outs[1] + u * 8) = pack8<T>(f);
  }
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace llmx_b200

using namespace llmx_b200;

extern "C" llmx_status llmx_attn_lse_merge(int32_t n_parts, const llmx_merge_part *parts, int32_t dtype,
                                           int32_t batch, int32_t seq, int32_t n_heads, int32_t head_dim, void *out,
                                           const int64_t *out_stride, float *lse_out, void *stream) {
  if (n_parts < 0 || n_parts > kMaxParts)
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: n_parts must be in [0, 16]");
  if (dtype != LLMX_FP16 && dtype != LLMX_BF16)
    return record_error(LLMX_ERR_UNSUPPORTED, "lse merge: dtype must be fp16 or bf16");
  if (batch < 1 || seq < 1 || n_heads < 1 || head_dim < 8 || head_dim % 8)
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: batch, seq, n_heads >= 1 and head_dim a multiple of 8");
  if (batch > 65535 || n_heads > 65535 || head_dim > 8192)
    return record_error(LLMX_ERR_INVALID_ARGUMENT,
                        "lse merge: batch and n_heads must be at most 65535, head_dim at most 8192");
  if (out == nullptr || out_stride == nullptr || !al16(out))
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: out and out_stride required, out 16-byte aligned");
  if (n_parts > 0 && parts == nullptr) return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: parts is NULL");
  MergeArgs m{};
  m.n_parts = n_parts;
  m.B = batch;
  m.S = seq;
  m.H = n_heads;
  m.D = head_dim;
  m.out = out;
  m.lse_out = lse_out;
  for (int i = 0; i < 3; ++i) {
    if (out_stride[i] < 0 || out_stride[i] % 8)
      return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: out strides must be >= 0 and multiples of 8");
    m.outs[i] = out_stride[i];
  }
  for (int c = 0; c < n_parts; ++c) {
    const llmx_merge_part &p = parts[c];
    if (p.row_lo < 0 || p.row_hi < p.row_lo || p.row_hi > seq)
      return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: part rows must satisfy 0 <= row_lo <= row_hi <= seq");
    if (p.row_hi > p.row_lo) {
      if (p.o == nullptr || p.lse == nullptr || !al16(p.o))
        return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: part o / lse required, o 16-byte aligned");
      for (int i = 0; i < 3; ++i)
        if (p.o_stride[i] < 0 || p.o_stride[i] % 8)
          return record_error(LLMX_ERR_INVALID_ARGUMENT,
                              "lse merge: part o strides must be >= 0 and multiples of 8");
      if (p.lse_stride[0] < 0 || p.lse_stride[1] < 0)
        return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: part lse strides must be >= 0");
    }
    PartDev &d = m.p[c];
    d.o = p.o;
    d.lse = p.lse;
    for (int i = 0; i < 3; ++i) d.os[i] = p.o_stride[i];
    d.ls[0] = p.lse_stride[0];
    d.ls[1] = p.lse_stride[1];
    d.row_lo = p.row_lo;
    d.row_hi = p.row_hi;
  }
  const int R = rows_of(head_dim);
  if ((seq + R - 1) / R > 65535)
    return record_error(LLMX_ERR_INVALID_ARGUMENT, "lse merge: seq too long for one launch (at most 65535 row runs)");
  const dim3 grid((unsigned)n_heads, (unsigned)((seq + R - 1) / R), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == LLMX_FP16)
    lse_merge_kernel<__half><<<grid, kMergeThreads, 0, st>>>(m);
  else
    lse_merge_kernel<__nv_bfloat16><<<grid, kMergeThreads, 0, st>>>(m);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LLMX_OK : record_error(LLMX_ERR_CUDA, cudaGetErrorString(e));
}
