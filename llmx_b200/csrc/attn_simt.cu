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
// Tiling: one CTA = 16 query rows of one (batch, head); 128 threads; key
// tiles of 64 staged in shared memory as fp32.
#include "common.cuh"

namespace llmx_b200 {
namespace {

constexpr int kBM = 16;
constexpr int kBN = 64;
constexpr int kThreads = 128;

template <int DMAX>
struct SimtSmem {
  static constexpr int kQ = kBM * DMAX;
  static constexpr int kK = kBN * (DMAX + 1);
  static constexpr int kV = kBN * DMAX;
  static constexpr int kS = kBM * kBN;
  static constexpr size_t bytes = sizeof(float) * (kQ + kK + kV + kS + 3 * kBM);
};

template <typename T, int DMAX>
__global__ void __launch_bounds__(kThreads) attn_simt_kernel(AttnArgs a) {
  extern __shared__ float smem[];
  float *Qs = smem;
  float *Ks = Qs + SimtSmem<DMAX>::kQ;
  float *Vs = Ks + SimtSmem<DMAX>::kK;
  float *Ss = Vs + SimtSmem<DMAX>::kV;
  float *m_s = Ss + SimtSmem<DMAX>::kS;
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

  // Q tile -> fp32 smem (rows past q_len and columns past D are zero).
  for (int e = tid; e < kBM * DMAX; e += kThreads) {
    const int r = e / DMAX, d = e % DMAX;
    const int qi = q0 + r;
    Qs[e] = (qi < ql && d < D) ? Elem<T>::to_f(qp[qi * a.qs[1] + d]) : 0.f;
  }
  if (tid < kBM) {
    m_s[tid] = -CUDART_INF_F;
    l_s[tid] = 0.f;
    alpha_s[tid] = 1.f;
  }

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

  // Output mapping: thread -> (row r_o, columns d_o + 8 i).
  const int r_o = tid / 8;
  const int d_o = tid % 8;
  constexpr int kPer = DMAX / 8;
  float acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
  __syncthreads();

  for (int n0 = lo; n0 < hi; n0 += kBN) {
    for (int e = tid; e < kBN * DMAX; e += kThreads) {
      const int c = e / DMAX, d = e % DMAX;
      const int j = n0 + c;
      const bool ok = j < kl && d < D;
      Ks[c * (DMAX + 1) + d] = ok ? Elem<T>::to_f(kp[j * a.ks[1] + d]) : 0.f;
      Vs[c * DMAX + d] = ok ? Elem<T>::to_f(vp[j * a.vs[1] + d]) : 0.f;
    }
    __syncthreads();
    // Scores: 16 x 64 entries, 8 per thread, lanes along keys.
    for (int e = tid; e < kBM * kBN; e += kThreads) {
      const int r = e / kBN, c = e % kBN;
      const int i = q0 + r, j = n0 + c;
      float s = -CUDART_INF_F;
      if (i < ql && key_visible(i, j, kl, doff, a.causal, a.window)) {
        float dot = 0.f;
        const float *qr = Qs + r * DMAX;
        const float *kr = Ks + c * (DMAX + 1);
        for (int d = 0; d < D; ++d) dot = fmaf(qr[d], kr[d], dot);
        s = score_transform(dot, a.sm_scale, a.softcap, slope, j + a.kv_offset);
      }
      Ss[e] = s;
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
        const float *vr = Vs + c * DMAX + d_o;
#pragma unroll
        for (int i = 0; i < kPer; ++i) acc[i] = fmaf(p, vr[8 * i], acc[i]);
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
      const int d = d_o + 8 * i;
      if (d < D) op[qi * a.os[1] + d] = Elem<T>::from_f(acc[i] * inv);
    }
    if (a.lse != nullptr && d_o == 0) {
      const float lse = (l > 0.f && qi < ql) ? m_s[r_o] + logf(l) : -CUDART_INF_F;
      a.lse[((long long)b * a.H + h) * a.Sq + qi] = lse;
    }
  }
}

template <typename T, int DMAX>
cudaError_t launch_simt_t(const AttnArgs &a, cudaStream_t s) {
  const size_t smem = SimtSmem<DMAX>::bytes;
  auto kern = attn_simt_kernel<T, DMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.Sq + kBM - 1) / kBM, a.H, a.B);
  kern<<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_simt_d(const AttnArgs &a, cudaStream_t s) {
  if (a.D <= 64) return launch_simt_t<T, 64>(a, s);
  if (a.D <= 128) return launch_simt_t<T, 128>(a, s);
  return launch_simt_t<T, 256>(a, s);
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
