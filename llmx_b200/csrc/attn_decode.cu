// Split-KV decode (one query row per sequence) and the log-sum-exp combine.
//
// Replaces the reference's decode path, which runs the prefill kernel with
// one 64-row tile per KV head (grid (1, n_kv_heads) per sequence,
// single_mha_kernel.cuh:630-634): 32 CTAs for a whole sequence leave most of
// a 148-SM part idle.  Here the key axis is cut into splits of `chunk` keys
// and every (split, kv head, batch) triple is a CTA, so the grid covers the
// machine whatever the batch; each CTA streams its K/V rows once with 16-byte
// non-allocating loads and keeps all query heads of its GQA group in
// registers (the reference packs the group into the M tile the same way,
// single_mha_kernel.cuh:434-441).
//
// Work split inside a CTA (128 threads): a key row of D halves is read by
// D/8 lanes (16 B each); a warp covers 32/(D/8) rows per step and unrolls 4
// steps, so each lane has 8 x 16 B of K and V in flight.  Dot products are
// reduced across the row's lanes with shuffles; the online softmax (running
// max m and sum l, softmax.h:53-110) runs per row group, then row groups and
// warps are merged.  With one split the CTA writes O directly; otherwise it
// writes a normalised partial (O_s, lse_s) and the combine kernel computes
//   lse = log sum_s exp(lse_s),  O = sum_s exp(lse_s - lse) O_s.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace llmx_b200 {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T, int D, int GP>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(AttnArgs a, int chunk, int n_splits,
                                                                 float *part_o, float *part_lse) {
  constexpr int LPR = D / 8;       // lanes per key row
  constexpr int RPW = 32 / LPR;    // key rows per warp step
  constexpr int KPW = RPW * kUnroll;  // keys per warp iteration
  constexpr int KPI = KPW * kWarps;   // keys per CTA iteration

  __shared__ float sm_m[kWarps][GP];
  __shared__ float sm_l[kWarps][GP];
  __shared__ float sm_acc[kWarps][GP][D];

  const int split = blockIdx.x;
  const int n_hgroups = (a.group + GP - 1) / GP;
  const int kvh = blockIdx.y / n_hgroups;
  const int hg = blockIdx.y % n_hgroups;
  const int b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int slot = lane % LPR;  // which 8 elements of the row
  const int rr = lane / LPR;    // which row of the warp step

  const int ql = clamp_len(a.q_lens, b, a.Sq);  // 0 or 1
  const int kl = ql > 0 ? clamp_len(a.kv_lens, b, a.Skv) : 0;
  const int k_begin = split * chunk;
  if (split > 0 && k_begin >= kl) return;  // nothing here; the combine skips it
  // The single query row sits on diagonal doff (local key index): causal
  // keys j <= doff, window keys j >= doff - window (mask.h:54-66).
  const int doff = diag_shift(a, 1, kl);
  int k_end = min(kl, k_begin + chunk);
  if (a.causal) k_end = min(k_end, max(k_begin, doff + 1));
  int k_lo = k_begin;
  if (a.window >= 0) k_lo = max(k_lo, doff - a.window);

  const int head0 = kvh * a.group + hg * GP;
  const int n_valid_heads = min(GP, a.group - hg * GP);

  // Query rows (one per head of the group slice) as fp32, this lane's slot.
  float qf[GP][8];
  float slope[GP];
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    const int h = head0 + (g < n_valid_heads ? g : 0);
    const T *qp = static_cast<const T *>(a.q) + b * a.qs[0] + h * a.qs[2] + slot * 8;
    uint4 u = *reinterpret_cast<const uint4 *>(qp);
    unpack8<T>(u, qf[g]);
    slope[g] = a.alibi ? a.alibi[h] * kLog2e : 0.f;
  }
  const float scale2 = a.sm_scale * kLog2e;  // scores kept in log2 units

  float m[GP], l[GP], acc[GP][8];
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    m[g] = -CUDART_INF_F;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }

  const char *kbase = reinterpret_cast<const char *>(static_cast<const T *>(a.k) + b * a.ks[0] +
                                                     kvh * a.ks[2] + slot * 8);
  const char *vbase = reinterpret_cast<const char *>(static_cast<const T *>(a.v) + b * a.vs[0] +
                                                     kvh * a.vs[2] + slot * 8);
  const long long kstep = a.ks[1] * (long long)sizeof(T);
  const long long vstep = a.vs[1] * (long long)sizeof(T);

  // Keys [k_lo, k_end) aligned down to the CTA iteration so that warps stay
  // in step; keys below k_lo are masked.
  const int it0 = k_begin + ((k_lo - k_begin) / KPI) * KPI;
  for (int base = it0; base < k_end; base += KPI) {
    uint4 kr[kUnroll], vr[kUnroll];
    int kj[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = base + warp * KPW + u * RPW + rr;
      kj[u] = j;
      if (j >= k_lo && j < k_end) {
        kr[u] = ld_stream16(kbase + j * kstep);
        vr[u] = ld_stream16(vbase + j * vstep);
      } else {
        kr[u] = make_uint4(0, 0, 0, 0);
        vr[u] = make_uint4(0, 0, 0, 0);
      }
    }
    float s[kUnroll][GP];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float kf[8];
      unpack8<T>(kr[u], kf);
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(qf[g][e], kf[e], d);
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        const bool vis = kj[u] >= k_lo && kj[u] < k_end;
        float sc;
        if (a.softcap > 0.f) {
          sc = tanhf(d * a.sm_scale / a.softcap) * a.softcap * kLog2e;
        } else {
          sc = d * scale2;
        }
        sc += slope[g] * (float)(kj[u] + a.kv_offset);
        s[u][g] = vis ? sc : -CUDART_INF_F;
      }
    }
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      float mx = s[0][g];
#pragma unroll
      for (int u = 1; u < kUnroll; ++u) mx = fmaxf(mx, s[u][g]);
      const float m_new = fmaxf(m[g], mx);
      if (m_new == -CUDART_INF_F) continue;  // nothing visible yet
      const float alpha = exp2f(m[g] - m_new);  // exp2(-inf) = 0
      float p[kUnroll];
      float ps = 0.f;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        p[u] = exp2f(s[u][g] - m_new);
        ps += p[u];
      }
      l[g] = l[g] * alpha + ps;
      m[g] = m_new;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float vf[8];
        unpack8<T>(vr[u], vf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p[u], vf[e], acc[g][e]);
      }
    }
  }

  // Merge the RPW row groups of the warp (lanes with the same slot).
#pragma unroll
  for (int off = LPR; off < 32; off <<= 1) {
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[g], off);
      const float mn = fmaxf(m[g], mo);
      const float a0 = (mn == -CUDART_INF_F) ? 0.f : exp2f(m[g] - mn);
      const float a1 = (mn == -CUDART_INF_F) ? 0.f : exp2f(mo - mn);
      l[g] = l[g] * a0 + lo * a1;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[g][e], off);
        acc[g][e] = acc[g][e] * a0 + ao * a1;
      }
      m[g] = mn;
    }
  }
  if (rr == 0) {
#pragma unroll
    for (int g = 0; g < GP; ++g) {
#pragma unroll
      for (int e = 0; e < 8; ++e) sm_acc[warp][g][slot * 8 + e] = acc[g][e];
      if (slot == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
    }
  }
  __syncthreads();

  // Merge warps: thread -> (head g, column d) pairs.
  for (int e = tid; e < GP * D; e += kThreads) {
    const int g = e / D, d = e % D;
    if (g >= n_valid_heads) continue;
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, sm_m[w][g]);
    float lsum = 0.f, o = 0.f;
    if (mx != -CUDART_INF_F) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float wt = exp2f(sm_m[w][g] - mx);
        lsum += sm_l[w][g] * wt;
        o += sm_acc[w][g][d] * wt;
      }
    }
    const int h = head0 + g;
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    const float lse = lsum > 0.f ? (mx + log2f(lsum)) * kLn2 : -CUDART_INF_F;
    if (n_splits == 1) {
      T *op = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
      op[d] = Elem<T>::from_f(o * inv);
      if (a.lse != nullptr && d == 0) a.lse[((long long)b * a.H + h) * a.Sq] = lse;
    } else {
      const long long row = ((long long)split * a.B + b) * a.H + h;
      part_o[row * D + d] = o * inv;
      if (d == 0) part_lse[row] = lse;
    }
  }
}

// O[b, 0, h, :] = sum_s exp(lse_s - lse) O_s over the splits that hold keys.
template <typename T, int D>
__global__ void __launch_bounds__(128) decode_combine_kernel(AttnArgs a, int chunk, int n_splits,
                                                              const float *part_o,
                                                              const float *part_lse) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int ql = clamp_len(a.q_lens, b, a.Sq);
  const int kl = ql > 0 ? clamp_len(a.kv_lens, b, a.Skv) : 0;
  const int n_used = max(1, min(n_splits, (kl + chunk - 1) / chunk));
  if (n_used <= 128) {
    // Up to 128 splits (one per thread): the split lse values are loaded
    // once, in parallel, and the weights exp(lse_s - max) go to shared
    // memory, so each output column is one pass of independent loads.  Same
    // expressions, in the same split order, as the general path below.
    __shared__ float w_s[128];
    __shared__ float red[4];
    const int tid = threadIdx.x;
    float l = -CUDART_INF_F;
    if (kl > 0 && tid < n_used) l = part_lse[((long long)tid * a.B + b) * a.H + h];
    float m = l;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (tid % 32 == 0) red[tid / 32] = m;
    __syncthreads();
    const float mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    if (tid < n_used) w_s[tid] = mx == -CUDART_INF_F ? 0.f : expf(l - mx);
    __syncthreads();
    float wsum = 0.f;
    if (mx != -CUDART_INF_F)
      for (int sidx = 0; sidx < n_used; ++sidx) wsum += w_s[sidx];
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    T *op = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
    for (int d = tid; d < D; d += blockDim.x) {
      float o = 0.f;
      if (wsum > 0.f) {
#pragma unroll 4
        for (int sidx = 0; sidx < n_used; ++sidx)
          o = fmaf(w_s[sidx], part_o[(((long long)sidx * a.B + b) * a.H + h) * D + d], o);
      }
      op[d] = Elem<T>::from_f(o * inv);
    }
    if (a.lse != nullptr && tid == 0)
      a.lse[((long long)b * a.H + h) * a.Sq] = wsum > 0.f ? mx + logf(wsum) : -CUDART_INF_F;
    return;
  }
  float mx = -CUDART_INF_F;
  if (kl > 0) {
    for (int sidx = 0; sidx < n_used; ++sidx)
      mx = fmaxf(mx, part_lse[((long long)sidx * a.B + b) * a.H + h]);
  }
  float wsum = 0.f;
  if (mx != -CUDART_INF_F) {
    for (int sidx = 0; sidx < n_used; ++sidx)
      wsum += expf(part_lse[((long long)sidx * a.B + b) * a.H + h] - mx);
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  T *op = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    if (wsum > 0.f) {
      for (int sidx = 0; sidx < n_used; ++sidx) {
        const long long row = ((long long)sidx * a.B + b) * a.H + h;
        o += expf(part_lse[row] - mx) * part_o[row * D + d];
      }
    }
    op[d] = Elem<T>::from_f(o * inv);
  }
  if (a.lse != nullptr && threadIdx.x == 0)
    a.lse[((long long)b * a.H + h) * a.Sq] = wsum > 0.f ? mx + logf(wsum) : -CUDART_INF_F;
}

template <typename T, int D, int GP>
cudaError_t launch_decode_t(const AttnArgs &a, const DecodePlan &p, void *ws, cudaStream_t s) {
  float *part_o = nullptr, *part_lse = nullptr;
  if (p.n_splits > 1) {
    part_o = static_cast<float *>(ws);
    part_lse = part_o + (size_t)p.n_splits * a.B * a.H * D;
  }
  const int n_hgroups = (a.group + GP - 1) / GP;
  dim3 grid(p.n_splits, a.Hkv * n_hgroups, a.B);
  decode_split_kernel<T, D, GP><<<grid, kThreads, 0, s>>>(a, p.chunk, p.n_splits, part_o, part_lse);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.n_splits == 1) return e;
  decode_combine_kernel<T, D><<<dim3(a.H, a.B), 128, 0, s>>>(a, p.chunk, p.n_splits, part_o, part_lse);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_decode_g(const AttnArgs &a, const DecodePlan &p, void *ws, cudaStream_t s) {
  switch (p.heads_per_cta) {
    case 1: return launch_decode_t<T, D, 1>(a, p, ws, s);
    case 2: return launch_decode_t<T, D, 2>(a, p, ws, s);
    case 4: return launch_decode_t<T, D, 4>(a, p, ws, s);
    default: return launch_decode_t<T, D, 8>(a, p, ws, s);
  }
}

template <typename T>
cudaError_t launch_decode_d(const AttnArgs &a, const DecodePlan &p, void *ws, cudaStream_t s) {
  switch (a.D) {
    case 64: return launch_decode_g<T, 64>(a, p, ws, s);
    case 128: return launch_decode_g<T, 128>(a, p, ws, s);
    case 256: return launch_decode_g<T, 256>(a, p, ws, s);
  }
  return cudaErrorNotSupported;
}

}  // namespace

DecodePlan plan_decode(const AttnArgs &a, size_t ws_available, bool have_ws) {
  DecodePlan p;
  const int g = a.group;
  p.heads_per_cta = g >= 8 ? 8 : (g >= 4 ? 4 : (g >= 2 ? 2 : 1));
  if (g > 1 && (g & (g - 1)) != 0 && g < 8) {
    // round a non power-of-two group up so one CTA holds all of it
    p.heads_per_cta = g <= 2 ? 2 : (g <= 4 ? 4 : 8);
  }
  const long long units = (long long)a.B * a.Hkv * ((g + p.heads_per_cta - 1) / p.heads_per_cta);
  // 256-key splits keep any one CTA's share of the stream short next to the
  // whole job; shorter splits when the batch alone cannot fill the machine.
  int chunk = 256;
  auto splits_for = [&](int c) { return (a.Skv + c - 1) / c; };
  while (chunk > 64 && units * splits_for(chunk) < 4LL * a.num_sms) chunk /= 2;
  int n = splits_for(chunk);
  if (n <= 1) {
    chunk = a.Skv;
    n = 1;
  }
  p.chunk = chunk;
  p.n_splits = n;
  p.ws_bytes = n > 1 ? (size_t)n * a.B * a.H * (a.D + 1) * sizeof(float) : 0;
  if (n > 1 && (!have_ws || ws_available < p.ws_bytes)) {
    p.chunk = a.Skv;
    p.n_splits = 1;
  }
  return p;
}

cudaError_t launch_decode(const AttnArgs &a, const DecodePlan &p, void *ws, cudaStream_t s) {
  switch (a.dtype) {
    case 1: return launch_decode_d<__half>(a, p, ws, s);
    case 2: return launch_decode_d<__nv_bfloat16>(a, p, ws, s);
  }
  return cudaErrorNotSupported;
}

}  // namespace llmx_b200

// ---------------------------------------------------------------------------
// Split-KV decode that allocates nothing.
//
// Some callers cannot call cudaMalloc or hand us a workspace: serving engines
// that fix their whole device-memory budget at start-up (KV cache, weights and
// activations reserved up front, any later allocation treated as a failure),
// and latency-critical loops that must not trigger cudaMalloc's implicit
// device-wide synchronisation.  For them the split partials live in a
// statically sized device array that this file owns.  Every GPU that loads
// the library holds the array until the process exits.
// ---------------------------------------------------------------------------
namespace llmx_b200 {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(LLMX_DECODE_NOALLOC_SCRATCH_BYTES);

// Host code must never use this name as a device address: on the host it is
// a stand-in object, so its address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxNoAllocDevices = 64;
float *g_noalloc_ptr[kMaxNoAllocDevices];
std::mutex g_noalloc_mu;

// Device address of the scratch array on `dev` (which must be current).
// Only a successful lookup is kept; a failed one (for example a first call
// made during stream capture) is retried by the next call.
// cudaGetSymbolAddress allocates nothing.
cudaError_t noalloc_scratch(int dev, float **out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();  // the failed lookup must not poison the next launch check
      *out = nullptr;
      return e;
    }
    if (p == nullptr) return cudaErrorInvalidSymbol;
    g_noalloc_ptr[dev] = static_cast<float *>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace llmx_b200

extern "C" llmx_status llmx_attn_decode_noalloc(const llmx_attn_params *p, void *stream) {
  using namespace llmx_b200;
  AttnArgs a;
  llmx_status s = prepare_decode_request(p, &a);
  if (s != LLMX_OK) return s;
  // Same split plan as llmx_attn_fwd with an unlimited workspace, so results
  // match it; requests whose partials exceed the array are refused.
  const DecodePlan plan = plan_decode(a, SIZE_MAX, true);
  if (plan.ws_bytes > kNoAllocScratchBytes) {
    char msg[200];
    snprintf(msg, sizeof msg,
             "llmx_attn_decode_noalloc: request needs %zu bytes of split-KV scratch; the static array "
             "holds %zu (LLMX_DECODE_NOALLOC_SCRATCH_BYTES)",
             plan.ws_bytes, kNoAllocScratchBytes);
    return record_error(LLMX_ERR_WORKSPACE_TOO_SMALL, msg);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxNoAllocDevices)
    return record_error(LLMX_ERR_NO_DEVICE, "llmx_attn_decode_noalloc: no usable current device");
  float *scratch = nullptr;
  cudaError_t e = noalloc_scratch(dev, &scratch);
  if (e != cudaSuccess)
    return record_error(LLMX_ERR_CUDA, "llmx_attn_decode_noalloc: cudaGetSymbolAddress failed");
  // Every partial the combine reads is written first by its split, so the
  // array's previous contents never need clearing.
  e = launch_decode(a, plan, scratch, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return record_error(LLMX_ERR_CUDA, cudaGetErrorString(e));
  return LLMX_OK;
}
