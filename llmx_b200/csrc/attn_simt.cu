// CUDA-core attention forward for every shape the engine accepts.
//
// This is the fp32 path (the CPU-runnable workload: B1 H8 S128 D64 fp32,
// causal, ALiBi) and the catch-all for fp16/bf16 requests outside the
// tensor-core kernels' envelope (head_dim not 64/128, unaligned strides).
// Arithmetic is fp32 throughout with accurate expf/tanhf, so fp32 inputs meet
// a 1e-4 max-abs bound against the fp32 oracle.
//
// Semantics follow the reference kernel's mainloop
// (single_mha_kernel.cuh:294-340): online softmax over key tiles with a
// running max/sum (softmax.h:53-145), bottom-right causal / window / length
// masks (mask.h:41-81) and ALiBi (mask.h:28-37,75-77).  Rows with no visible
// key produce 0 instead of the reference's NaN.
//
// Tiling: one CTA = kBM (16, or 8 when 16-row tiles would leave SMs idle)
// query rows of one (batch, head); 128 threads; key tiles of 64 staged in
// shared memory as fp32.  Small problems are latency-bound, so the staging
// of Q, K and V tiles issues a thread's 16-byte loads in batches of four
// before converting and storing any of them (rows with 16-byte aligned
// starts; other layouts take element loads).
#include "common.cuh"

namespace llmx_b200 {
namespace {

constexpr int kBN = 64;
constexpr int kThreads = 128;

// Row pitch of the K tile in shared memory: 16-byte aligned rows, and the
// 4-word skew spreads the 16-byte reads of lanes on consecutive rows over
// all 32 banks.
template <int DMAX>
constexpr int kKPitch = DMAX + 4;

template <int DMAX, int kBM>
struct SimtSmem {
  static constexpr int kQ = kBM * DMAX;
  static constexpr int kK = kBN * kKPitch<DMAX>;
  static constexpr int kV = kBN * DMAX;
  static constexpr int kS = kBM * kBN;
  static constexpr size_t bytes = sizeof(float) * (kQ + kK + kV + kS + 3 * kBM);
};

// 16 bytes of T -> floats (4 for fp32, 8 for 16-bit types).
template <typename T>
__device__ __forceinline__ void unpack16(const uint4 &u, float *f) {
  if constexpr (std::is_same<T, float>::value) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    float g[8];
    unpack8<T>(u, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = g[i];
  }
}

// Stages rows [r0, r0 + n_rows) (row r at src + r * stride, D elements) into
// dst[(r - r0) * dst_pitch + d] as fp32; rows at or past `valid` and columns
// past D are zero.  vec: 16-byte aligned row starts and D a multiple of the
// 16-byte element count.
template <typename T, int DMAX>
__device__ __forceinline__ void stage_rows(float *dst, int dst_pitch, const T *src, long long stride, int r0,
                                           int n_rows, int valid, int D, bool vec) {
  constexpr int kE = 16 / sizeof(T);  // elements per 16-byte unit
  if (vec) {
    const int upr = DMAX / kE;  // units per staged row (columns past D read as zero)
    const int n_units = n_rows * upr;
    for (int base = threadIdx.x; base < n_units; base += 4 * kThreads) {
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * kThreads;
        const int r = idx / upr, x = idx - r * upr;
        raw[u] = make_uint4(0u, 0u, 0u, 0u);
        if (idx < n_units && r0 + r < valid && x * kE < D)
          raw[u] = *reinterpret_cast<const uint4 *>(src + (long long)(r0 + r) * stride + x * kE);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * kThreads;
        if (idx < n_units) {
          const int r = idx / upr, x = idx - r * upr;
          float f[kE];
          unpack16<T>(raw[u], f);
#pragma unroll
          for (int i = 0; i < kE; ++i) dst[r * dst_pitch + x * kE + i] = f[i];
        }
      }
    }
  } else {
    for (int e = threadIdx.x; e < n_rows * DMAX; e += kThreads) {
      const int r = e / DMAX, d = e % DMAX;
      dst[r * dst_pitch + d] = (r0 + r < valid && d < D) ? Elem<T>::to_f(src[(long long)(r0 + r) * stride + d]) : 0.f;
    }
  }
}

// Stages key rows [n0, n0 + kBN) of K (pitch kKPitch) and V (pitch DMAX)
// together: with 16-byte rows every thread issues all of its K and V loads
// of the tile (up to 16) before storing any, so the tile costs one memory
// round trip instead of one per load.
template <typename T, int DMAX>
__device__ __forceinline__ void stage_kv(float *Ks, float *Vs, const T *kp, const T *vp, long long ks, long long vs,
                                         int n0, int valid, int D, bool vec) {
  constexpr int kE = 16 / sizeof(T);
  constexpr int kUpr = DMAX / kE;                    // 16-byte units per row
  constexpr int kUnits = kBN * kUpr;                 // per tensor
  constexpr int kPer = kUnits / kThreads;            // per thread and tensor
  constexpr int kBatch = kPer < 8 ? kPer : 8;        // loads per tensor in flight
  static_assert(kUnits % kThreads == 0 && kPer % kBatch == 0, "tile shape");
  if (!vec) {
    stage_rows<T, DMAX>(Ks, kKPitch<DMAX>, kp, ks, n0, kBN, valid, D, false);
    stage_rows<T, DMAX>(Vs, DMAX, vp, vs, n0, kBN, valid, D, false);
    return;
  }
#pragma unroll 1
  for (int b0 = 0; b0 < kPer; b0 += kBatch) {
    uint4 rk[kBatch], rv[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int idx = threadIdx.x + (b0 + u) * kThreads;
      const int r = idx / kUpr, x = idx - r * kUpr;
      rk[u] = rv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (n0 + r < valid && x * kE < D) {
        rk[u] = *reinterpret_cast<const uint4 *>(kp + (long long)(n0 + r) * ks + x * kE);
        rv[u] = *reinterpret_cast<const uint4 *>(vp + (long long)(n0 + r) * vs + x * kE);
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int idx = threadIdx.x + (b0 + u) * kThreads;
      const int r = idx / kUpr, x = idx - r * kUpr;
      float f[kE];
      unpack16<T>(rk[u], f);
#pragma unroll
      for (int i = 0; i < kE; ++i) Ks[r * kKPitch<DMAX> + x * kE + i] = f[i];
      unpack16<T>(rv[u], f);
#pragma unroll
      for (int i = 0; i < kE; ++i) Vs[r * DMAX + x * kE + i] = f[i];
    }
  }
}

// A key tile held in registers between its loads and its shared-memory
// stores, so the next tile's loads can be in flight while the current tile
// is computed (layouts with 16-byte rows whose tile is one batch of loads:
// kPer <= 8 units per thread and tensor).
template <typename T, int DMAX>
struct KVPrefetch {
  static constexpr int kE = 16 / sizeof(T);
  static constexpr int kUpr = DMAX / kE;
  static constexpr int kPer = kBN * kUpr / kThreads;
  static constexpr bool kUsable = kPer <= 8 && kPer * kThreads == kBN * kUpr;
  uint4 rk[kPer], rv[kPer];

  __device__ __forceinline__ void load(const T *kp, const T *vp, long long ks, long long vs, int n0, int valid,
                                       int D) {
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int idx = threadIdx.x + u * kThreads;
      const int r = idx / kUpr, x = idx - r * kUpr;
      rk[u] = rv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (n0 + r < valid && x * kE < D) {
        rk[u] = *reinterpret_cast<const uint4 *>(kp + (long long)(n0 + r) * ks + x * kE);
        rv[u] = *reinterpret_cast<const uint4 *>(vp + (long long)(n0 + r) * vs + x * kE);
      }
    }
  }
  __device__ __forceinline__ void store(float *Ks, float *Vs) const {
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int idx = threadIdx.x + u * kThreads;
      const int r = idx / kUpr, x = idx - r * kUpr;
      float f[kE];
      unpack16<T>(rk[u], f);
#pragma unroll
      for (int i = 0; i < kE; ++i) Ks[r * kKPitch<DMAX> + x * kE + i] = f[i];
      unpack16<T>(rv[u], f);
#pragma unroll
      for (int i = 0; i < kE; ++i) Vs[r * DMAX + x * kE + i] = f[i];
    }
  }
};

template <typename T, int DMAX, int kBM>
__global__ void __launch_bounds__(kThreads) attn_simt_kernel(AttnArgs a, bool vec) {
  using Sm = SimtSmem<DMAX, kBM>;
  constexpr int kCols = kThreads / kBM;  // output column groups per row
  extern __shared__ float smem[];
  float *Qs = smem;
  float *Ks = Qs + Sm::kQ;
  float *Vs = Ks + Sm::kK;
  float *Ss = Vs + Sm::kV;
  float *m_s = Ss + Sm::kS;
  float *l_s = m_s + kBM;
  float *alpha_s = l_s + kBM;

  const int tid = threadIdx.x;
  const int q0 = blockIdx.x * kBM;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int D = a.D;
  const int kvh = h / a.group;
  const int ql = clamp_len(a.q_lens, b, a.Sq);
  const int kl = clamp_len(a.kv_lens, b, a.Skv);
  const T *qp = static_cast<const T *>(a.q) + b * a.qs[0] + h * a.qs[2];
  const T *kp = static_cast<const T *>(a.k) + b * a.ks[0] + kvh * a.ks[2];
  const T *vp = static_cast<const T *>(a.v) + b * a.vs[0] + kvh * a.vs[2];
  T *op = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
  const float slope = a.alibi ? a.alibi[h] : 0.f;

  // Key range that any row of this tile can see.
  const int doff = diag_shift(a, ql, kl);
  const int r_last = min(q0 + kBM, ql) - 1;
  int lo = 0, hi = kl;
  if (q0 < ql) {
    if (a.causal) hi = max(0, min(kl, r_last + doff + 1));
    if (a.window >= 0) lo = min(kl, max(0, q0 + doff - a.window));
  } else {
    hi = 0;
  }
  lo = (lo / kBN) * kBN;

  // The first key tile's loads are issued before the Q tile is staged, so
  // the two memory round trips overlap.
  using Pf = KVPrefetch<T, DMAX>;
  Pf pf;
  const bool prefetch = Pf::kUsable && vec;
  if (prefetch && lo < hi) pf.load(kp, vp, a.ks[1], a.vs[1], lo, kl, D);

  // Q tile -> fp32 smem (rows past q_len and columns past D are zero).
  stage_rows<T, DMAX>(Qs, DMAX, qp, a.qs[1], q0, kBM, ql, D, vec);
  if (tid < kBM) {
    m_s[tid] = -CUDART_INF_F;
    l_s[tid] = 0.f;
    alpha_s[tid] = 1.f;
  }

  // Output mapping: thread -> row r_o, columns 4 d_o + 4 kCols g + (0..3)
  // for g < kPer / 4 (one 16-byte read of a V row per group and key).
  const int r_o = tid / kCols;
  const int d_o = tid % kCols;
  constexpr int kPer = DMAX / kCols;
  static_assert(kPer % 4 == 0, "four consecutive output columns per group");
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
  __syncthreads();

  for (int n0 = lo; n0 < hi; n0 += kBN) {
    if (prefetch) {
      pf.store(Ks, Vs);
      // the next tile's loads fly while this one is computed
      if (n0 + kBN < hi) pf.load(kp, vp, a.ks[1], a.vs[1], n0 + kBN, kl, D);
    } else {
      stage_kv<T, DMAX>(Ks, Vs, kp, vp, a.ks[1], a.vs[1], n0, kl, D, vec);
    }
    __syncthreads();
    // Scores: kBM x kBN entries; thread t takes key column c = t % kBN of
    // kSc rows (t / kBN + g * kThreads / kBN), so one 16-byte read of its K
    // row feeds kSc independent dot products (Q reads are warp broadcasts).
    // Columns past D are zero in both tiles, so the sums over DMAX equal
    // the sums over D, accumulated in the same order.
    {
      constexpr int kSc = kBM * kBN / kThreads;
      static_assert(kThreads % kBN == 0, "one key column per thread");
      const int c = tid % kBN;
      const int rb = tid / kBN;
      float dot[kSc];
#pragma unroll
      for (int g = 0; g < kSc; ++g) dot[g] = 0.f;
      const float *kr = Ks + c * kKPitch<DMAX>;
#pragma unroll 4
      for (int d = 0; d < DMAX; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4 *>(kr + d);
#pragma unroll
        for (int g = 0; g < kSc; ++g) {
          const float4 q4 = *reinterpret_cast<const float4 *>(Qs + (rb + g * (kThreads / kBN)) * DMAX + d);
          dot[g] = fmaf(q4.x, k4.x, dot[g]);
          dot[g] = fmaf(q4.y, k4.y, dot[g]);
          dot[g] = fmaf(q4.z, k4.z, dot[g]);
          dot[g] = fmaf(q4.w, k4.w, dot[g]);
        }
      }
#pragma unroll
      for (int g = 0; g < kSc; ++g) {
        const int r = rb + g * (kThreads / kBN);
        const int i = q0 + r, j = n0 + c;
        float s = -CUDART_INF_F;
        if (i < ql && key_visible(i, j, kl, doff, a.causal, a.window))
          s = score_transform(dot[g], a.sm_scale, a.softcap, slope, j + a.kv_offset);
        Ss[r * kBN + c] = s;
      }
    }
    __syncthreads();
    // Online softmax: warp w owns rows 4w .. 4w+3.
    {
      const int w = tid / 32, lane = tid % 32;
      for (int rr = 0; rr < kBM / 4; ++rr) {
        const int r = w * (kBM / 4) + rr;
        float s0 = Ss[r * kBN + lane], s1 = Ss[r * kBN + lane + 32];
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float m_old = m_s[r];
        const float m_new = fmaxf(m_old, mx);
        const float m_use = (m_new == -CUDART_INF_F) ? 0.f : m_new;
        const float p0 = expf(s0 - m_use), p1 = expf(s1 - m_use);
        float ps = p0 + p1;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        Ss[r * kBN + lane] = p0;
        Ss[r * kBN + lane + 32] = p1;
        __syncwarp();
        if (lane == 0) {
          const float alpha = (m_old == -CUDART_INF_F) ? 0.f : expf(m_old - m_use);
          alpha_s[r] = alpha;
          l_s[r] = l_s[r] * alpha + ps;
          m_s[r] = m_new;
        }
      }
    }
    __syncthreads();
    {
      const float alpha = alpha_s[r_o];
      const float *pr = Ss + r_o * kBN;
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc[i] *= alpha;
      for (int c = 0; c < kBN; ++c) {
        const float p = pr[c];
        const float *vr = Vs + c * DMAX + 4 * d_o;
#pragma unroll
        for (int g = 0; g < kPer / 4; ++g) {
          const float4 v4 = *reinterpret_cast<const float4 *>(vr + 4 * kCols * g);
          acc[4 * g] = fmaf(p, v4.x, acc[4 * g]);
          acc[4 * g + 1] = fmaf(p, v4.y, acc[4 * g + 1]);
          acc[4 * g + 2] = fmaf(p, v4.z, acc[4 * g + 2]);
          acc[4 * g + 3] = fmaf(p, v4.w, acc[4 * g + 3]);
        }
      }
    }
    __syncthreads();
  }

  const int qi = q0 + r_o;
  if (qi < a.Sq) {
    const float l = l_s[r_o];
    const float inv = (l > 0.f && qi < ql) ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = 4 * d_o + 4 * kCols * (i / 4) + (i % 4);
      if (d < D) op[qi * a.os[1] + d] = Elem<T>::from_f(acc[i] * inv);
    }
    if (a.lse != nullptr && d_o == 0) {
      const float lse = (l > 0.f && qi < ql) ? m_s[r_o] + logf(l) : -CUDART_INF_F;
      a.lse[((long long)b * a.H + h) * a.Sq + qi] = lse;
    }
  }
}

template <typename T, int DMAX, int kBM>
cudaError_t launch_simt_t(const AttnArgs &a, bool vec, cudaStream_t s) {
  const size_t smem = SimtSmem<DMAX, kBM>::bytes;
  auto kern = attn_simt_kernel<T, DMAX, kBM>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((a.Sq + kBM - 1) / kBM, a.H, a.B);
  kern<<<grid, kThreads, smem, s>>>(a, vec);
  return cudaGetLastError();
}

// 16-row tiles, or 8-row tiles when 16-row tiles leave SMs without a CTA.
template <typename T, int DMAX>
cudaError_t launch_simt_m(const AttnArgs &a, bool vec, cudaStream_t s) {
  const long long ctas16 = (long long)((a.Sq + 15) / 16) * a.H * a.B;
  if (ctas16 < a.num_sms) return launch_simt_t<T, DMAX, 8>(a, vec, s);
  return launch_simt_t<T, DMAX, 16>(a, vec, s);
}

template <typename T>
cudaError_t launch_simt_d(const AttnArgs &a, cudaStream_t s) {
  constexpr int kE = 16 / sizeof(T);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  bool vec = al16(a.q) && al16(a.k) && al16(a.v) && a.D % kE == 0;
  for (int i = 1; i < 3; ++i) vec = vec && a.qs[i] % kE == 0 && a.ks[i] % kE == 0 && a.vs[i] % kE == 0;
  vec = vec && a.qs[0] % kE == 0 && a.ks[0] % kE == 0 && a.vs[0] % kE == 0;
  if (a.D <= 64) return launch_simt_m<T, 64>(a, vec, s);
  if (a.D <= 128) return launch_simt_m<T, 128>(a, vec, s);
  return launch_simt_m<T, 256>(a, vec, s);
}

}  // namespace

cudaError_t launch_simt(const AttnArgs &a, cudaStream_t s) {
  switch (a.dtype) {
    case 0: return launch_simt_d<float>(a, s);
    case 1: return launch_simt_d<__half>(a, s);
    case 2: return launch_simt_d<__nv_bfloat16>(a, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace llmx_b200
