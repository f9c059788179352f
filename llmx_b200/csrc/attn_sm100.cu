// Fused attention forward on Blackwell tensor cores (sm_100a): TMA-staged
// Q/K/V tiles, S = QK^T and O += PV on tcgen05.mma with both accumulators in
// tensor memory, and scale + soft-cap + ALiBi + causal / window / length
// masks + online softmax fused between the two GEMMs.  Scores never leave
// the SM.
//
// Reference path replaced: SingleMHACollectiveMainloop + SingleMHAKernel
// (include/llmx/cuda/attention/device/single_mha_kernel.cuh:30-345,479-593),
// an SM80 mma.sync kernel with a 64x64 tile, one cp.async stage and
// register-resident accumulators.  Semantics kept: bottom-right causal
// alignment and window (mask.h:41-81), ALiBi as + slope*j (mask.h:75-77),
// soft-cap tanh(s*scale/cap)*cap (params.h:35-50), P rounded to the input
// type before PV (single_mha_kernel.cuh:232-233), GQA head h -> kv head
// h / group.
//
// CTA = 2 query tiles of 128 rows of one (batch, head); 12 warps:
//   warps 0-3   softmax for query tile 0 (thread r owns row r = TMEM lane r)
//   warps 4-7   softmax for query tile 1
//   warp  8     tensor-memory allocation + MMA issue (one thread)
//   warp  9     TMA producer (one thread)
//   warps 10-11 idle (they complete the third warpgroup for setmaxnreg)
// Tensor memory (512 columns x 128 lanes of 32 bit):
//   [0,128) S0 / P0, [128,256) S1 / P1, [256,256+D) O0, [256+D,256+2D) O1.
// P (16-bit, two per column) overwrites the first 64 columns of its S.
//
// Per KV block j of 128 keys the MMA thread issues, in order,
//   O0 += P0(j) V(j),   S0(j+1) = Q0 K(j+1)^T,   O1 += P1(j) V(j),   S1(j+1)
// so each softmax warpgroup's exponentials overlap the other tile's GEMMs;
// tcgen05 operations from one thread execute in issue order, which is what
// lets S0(j+1) overwrite P0(j) right after PV0(j) is issued.  With ALiBi the
// key blocks are taken last to first (block_n0), as in the reference.
//
// Online softmax: running max m and sum l per row in log2 units.  The max is
// only moved (and O rescaled in tensor memory) when a block raises it by more
// than rescale_threshold (2^64 for bf16, 2^15 for fp16), so O rescales are
// rare; the final O / l is the same softmax.
//
// Every mbarrier wait is bounded (1 s); on expiry the kernel records
// kDevErrTimeout in the device error word, unwinds all roles, waits (bounded)
// for its in-flight TMA loads and MMAs, frees tensor memory and exits.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace llmx_b200 {
namespace {

using namespace sm100;

constexpr int kBM = 128;       // query rows per tile
constexpr int kTiles = 2;      // query tiles per CTA
constexpr int kBN = 128;       // keys per KV block
constexpr int kThreads = 384;  // 2 softmax warpgroups + MMA / TMA warpgroup
constexpr int kMmaWarp = 8;
constexpr int kTmaWarp = 9;
// Register split (setmaxnreg, multiples of 8): the CTA launches with 384 x 168;
// the MMA / TMA warpgroup drops to 64 and the softmax warpgroups grow to 216:
// 128 * 64 + 256 * 216 = 63488 <= 384 * 168 = 64512.
constexpr uint32_t kRegsControl = 64;
constexpr uint32_t kRegsSoftmax = 216;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * 168, "register split exceeds the launch");
constexpr uint64_t kTimeoutNs = 1000000000ull;
constexpr int kSchedSlots = 4;
constexpr int kSchedConsumers = 1 + 8;  // the MMA thread + one lane per softmax warp
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// Lazy rescale: the running max moves (and O is rescaled) only when a block
// raises it by more than this many log2 units, so P <= 2^threshold.  bf16 P
// has the fp32 exponent range and O / l accumulate in fp32, so 2^64; fp16 P
// must stay below 65504, so 2^15.
template <typename T>
constexpr float rescale_threshold() {
  return std::is_same<T, __nv_bfloat16>::value ? 64.0f : 15.0f;
}

template <int D>
struct Cfg {
  static constexpr int kChunks = D / 64;          // 128-byte wide column chunks of a tile
  static constexpr int kChunkBytes = 128 * 128;   // 128 rows x 128 bytes
  static constexpr int kTileBytes = 128 * D * 2;  // one 128-row tile of 16-bit elements
  static constexpr int kStages = D == 128 ? 2 : 3;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kTiles * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  // ALiBi operands of the extra QK^T step (K-major, no swizzle, 4 KB used
  // of 8 KB each): A' per query tile, B' shared.
  static constexpr int kXOff = kVOff + kStages * kTileBytes;
  static constexpr int kXBytes = 8192;
  static constexpr int kBarOff = kXOff + 3 * kXBytes;
  static constexpr int kSmemBytes = kBarOff + 1024 + 1024;  // barriers + alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  static constexpr uint32_t kTmemS0 = 0, kTmemS1 = 128;
  static constexpr uint32_t kTmemO0 = 256, kTmemO1 = 256 + D;
  static constexpr uint32_t kTmemCols = 512;
};

// A decoded work item as the TMA thread publishes it in the ring (the
// consumers copy it instead of each decoding the index again).
struct ItemPod {
  int h, b, kvh, ql, kl, m0, n_start, nb, nb0;
};

struct Bars {
  uint64_t q_full[2], q_empty[2];  // one per query tile
  uint64_t k_full[3], k_empty[3], v_full[3], v_empty[3];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint64_t drain;
  // Work-item ring: the TMA thread publishes each item index (and finally an
  // index >= n_work) to the MMA thread and the eight softmax warps.
  uint64_t sched_full[kSchedSlots], sched_empty[kSchedSlots];
  int sched_w[kSchedSlots];
  ItemPod sched_item[kSchedSlots];
  uint32_t tmem_base;
  volatile int abort_flag;
};

template <typename B>
__device__ __forceinline__ void set_abort(B *bars, unsigned int *err) {
  bars->abort_flag = 1;
  raise_error(err, kDevErrTimeout);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  }
}

// Key-block range of the CTA: blocks [n_start, n_start + nb*kBN).
struct BlockRange {
  int n_start, nb;
};

// First key of the j-th block processed.  With ALiBi the blocks go last to
// first, as the reference's main loop does (single_mha_kernel.cuh:295-296):
// the bias slope * key grows with the key, so the first block processed
// holds the row's largest biases, the running max is set there, and later
// blocks rarely raise it (each raise rescales O).
template <bool kReverse>
__device__ __forceinline__ int block_n0(const BlockRange &br, int j) {
  return br.n_start + (kReverse ? br.nb - 1 - j : j) * kBN;
}

// rows: query rows per work item (kTiles * kBM, or kBM for head_dim 256).
__device__ __forceinline__ BlockRange block_range(const AttnArgs &a, int m0, int ql, int kl, int rows) {
  BlockRange r{0, 0};
  if (m0 >= ql || kl <= 0) return r;
  const int off = diag_shift(a, ql, kl);
  const int r_last = min(m0 + rows, ql) - 1;
  const int hi = a.causal ? min(kl, r_last + off + 1) : kl;
  int lo = a.window >= 0 ? max(0, m0 + off - a.window) : 0;
  lo = (lo / kBN) * kBN;
  if (hi > lo) {
    r.n_start = lo;
    r.nb = (hi - lo + kBN - 1) / kBN;
  }
  return r;
}

// One work item: a (batch, head) unit and a pair of 128-row query tiles.
struct Work {
  int h, b, kvh, ql, kl, m0;
  BlockRange br;  // key blocks of the item (all visible to tile 1)
  int nb0;        // leading blocks of br that tile 0 (the earlier rows) sees, >= 1
};

// Work item w in the launch's order: (batch, head) units in groups of
// `group_units` whose K/V fit in L2 together; inside a group the query-tile
// pairs go longest first (with causal masking the highest rows see the most
// keys), so the machine works on one L2-resident K/V set at a time and short
// items fill the tail.
__device__ __forceinline__ Work decode_work(const AttnArgs &a, int w, int n_mblocks, int group_units,
                                            int rows = kTiles * kBM) {
  const int units = a.B * a.H;
  const int per_group = group_units * n_mblocks;
  const int g = w / per_group;
  const int within = w - g * per_group;
  const int gu = min(group_units, units - g * group_units);
  const int rank = within / gu;
  const int unit = g * group_units + within % gu;
  const int mblk = a.causal ? (n_mblocks - 1 - rank) : rank;
  Work t;
  t.h = unit % a.H;
  t.b = unit / a.H;
  t.kvh = t.h / a.group;
  t.ql = clamp_len(a.q_lens, t.b, a.Sq);
  t.kl = clamp_len(a.kv_lens, t.b, a.Skv);
  t.m0 = mblk * rows;
  t.br = block_range(a, t.m0, t.ql, t.kl, rows);
  t.nb0 = t.br.nb;
  if (a.causal && t.br.nb > 0) {
    // With causal masking tile 0's last visible key is row m0 + 127's
    // diagonal; blocks past it are skipped for tile 0 (at least one is kept).
    const int hi0 = min(t.kl, min(t.m0 + kBM, t.ql) + diag_shift(a, t.ql, t.kl));
    t.nb0 = max(1, min(t.br.nb, (hi0 - t.br.n_start + kBN - 1) / kBN));
  }
  return t;
}

// Scheduling.  CTA i starts with item i; with a work counter (persistent
// launch, one CTA per SM) the TMA thread then takes item G + atomicAdd(ctr, 1)
// each time it finishes issuing the loads of one, so CTAs that drew short
// items take more of them; without one (one CTA per item) it stops after
// its first.  Every item index, and a final one >= n_work, goes through the
// shared-memory ring to the other roles, so all roles see the same sequence;
// the main kernel's ring slots also carry the decoded item (sched_publish_item
// / sched_take_item), which saves the MMA thread and the eight softmax warps
// the integer divisions of decode_work at every item boundary.
template <typename B>
__device__ __forceinline__ bool sched_publish(B *bars, int n, int w) {
  const int slot = n % kSchedSlots;
  if (n >= kSchedSlots &&
      !mbar_wait_or_abort(&bars->sched_empty[slot], ((n / kSchedSlots) - 1) & 1, kTimeoutNs, &bars->abort_flag))
    return false;
  bars->sched_w[slot] = w;
  mbar_arrive(&bars->sched_full[slot]);  // release: orders the store above
  return true;
}
__device__ __forceinline__ bool sched_publish_item(Bars *bars, int n, int w, const Work &t) {
  const int slot = n % kSchedSlots;
  if (n >= kSchedSlots &&
      !mbar_wait_or_abort(&bars->sched_empty[slot], ((n / kSchedSlots) - 1) & 1, kTimeoutNs, &bars->abort_flag))
    return false;
  bars->sched_w[slot] = w;
  ItemPod &it = bars->sched_item[slot];
  it.h = t.h; it.b = t.b; it.kvh = t.kvh; it.ql = t.ql; it.kl = t.kl; it.m0 = t.m0;
  it.n_start = t.br.n_start; it.nb = t.br.nb; it.nb0 = t.nb0;
  mbar_arrive(&bars->sched_full[slot]);  // release: orders the stores above
  return true;
}
// sched_take that also copies the published item (valid when w < n_work).
__device__ __forceinline__ int sched_take_item(Bars *bars, int n, bool warp_wide, Work &t) {
  const int slot = n % kSchedSlots;
  bool ok = mbar_wait_or_abort(&bars->sched_full[slot], (n / kSchedSlots) & 1, kTimeoutNs, &bars->abort_flag);
  if (warp_wide) ok = __all_sync(0xffffffffu, ok);
  if (!ok) return -1;
  const int w = *reinterpret_cast<volatile int *>(&bars->sched_w[slot]);
  const volatile ItemPod &it = bars->sched_item[slot];
  t.h = it.h; t.b = it.b; t.kvh = it.kvh; t.ql = it.ql; t.kl = it.kl; t.m0 = it.m0;
  t.br.n_start = it.n_start; t.br.nb = it.nb; t.nb0 = it.nb0;
  if (warp_wide) __syncwarp();
  if (!warp_wide || (threadIdx.x % 32) == 0) mbar_arrive(&bars->sched_empty[slot]);
  return w;
}

// The n-th item of the sequence for a consumer role, or -1 on abort.  One
// thread per consumer (the MMA thread, lane 0 of each softmax warp) arrives
// on sched_empty once every thread it stands for has read the slot.
template <typename B>
__device__ __forceinline__ int sched_take(B *bars, int n, bool warp_wide) {
  const int slot = n % kSchedSlots;
  bool ok = mbar_wait_or_abort(&bars->sched_full[slot], (n / kSchedSlots) & 1, kTimeoutNs, &bars->abort_flag);
  if (warp_wide) ok = __all_sync(0xffffffffu, ok);
  if (!ok) return -1;
  const int w = *reinterpret_cast<volatile int *>(&bars->sched_w[slot]);
  if (warp_wide) __syncwarp();
  if (!warp_wide || (threadIdx.x % 32) == 0) mbar_arrive(&bars->sched_empty[slot]);
  return w;
}

// ALiBi folded into QK^T (no soft-cap): one more K = 16 step adds
// beta * c to S[r][c], beta = slope / sm_scale, c = the key's column in its
// 128-key block.  A'_t (128 x 16, per query tile) holds beta as three 16-bit
// parts in columns 0-2 of every row; B' (128 x 16) holds c in columns 0-2 of
// row c.  Integers below 256 are exact in both 16-bit types and the products
// are exact in fp32, so S' = S + beta * c to fp32 rounding.  The softmax then
// treats ALiBi like the plain path plus slope * (n0 + kv_offset) per block.
// Byte offset of element (r, k) in the no-swizzle K-major layout used for
// A' and B': 8-row x 16-byte core matrices, 128 bytes apart along K,
// 256 bytes apart between 8-row groups.
__device__ __forceinline__ int x_offset(int r, int k) {
  return (r >> 3) * 256 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
}

// Loads issued so far by the TMA thread (for the drain before exit).
struct TmaCounts {
  int k = 0, v = 0, q[2] = {0, 0};
};

// ---------------------------------------------------------------- TMA role
// Loads for one work item: Q tile 0, then per key block K (and after the
// first K, Q tile 1) and V through the ring.  kv_base is the number of key
// blocks of earlier items (ring position and phase); a Q buffer is refilled
// once the previous item's last QK^T on it has completed (q_empty).
// With kFold the thread also writes the item's ALiBi row (beta: the slope
// over sm_scale as three 16-bit parts) into A'_q before signalling Q_q.
// The Q load is issued before A'_q is written (the tile's bytes are added
// to q_full first, the thread's arrival comes after the A' stores), so the
// load's latency overlaps the slope read and the stores.
template <typename T, int D, bool kFold, bool kReverse>
__device__ bool tma_tile(const CUtensorMap *tm_q, const CUtensorMap *tm_k, const CUtensorMap *tm_v, uint8_t *smem,
                         Bars *bars, const Work &t, int tile_it, int kv_base, TmaCounts &n, const AttnArgs &a) {
  using C = Cfg<D>;
  auto wait = [&](uint64_t *bar, uint32_t par) {
    return mbar_wait_or_abort(bar, par, kTimeoutNs, &bars->abort_flag);
  };
  uint4 beta = make_uint4(0u, 0u, 0u, 0u);
  auto load_q = [&](int q) {
    if (tile_it > 0 && !wait(&bars->q_empty[q], (tile_it - 1) & 1)) return false;
    mbar_expect_tx(&bars->q_full[q], C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_4d(smem + C::kQOff + q * C::kTileBytes + c * C::kChunkBytes, tm_q, &bars->q_full[q], c * 64, t.h,
                  t.m0 + q * kBM, t.b);
    if constexpr (kFold) {
      if (q == 0) {
        // beta = slope / sm_scale as three 16-bit parts (each the rounding
        // of what the previous ones leave), in columns 0-2.
        const float b = a.alibi[t.h] / a.sm_scale;
        const float r1 = b - Elem<T>::to_f(Elem<T>::from_f(b));
        const float r2 = r1 - Elem<T>::to_f(Elem<T>::from_f(r1));
        const float f[8] = {b, r1, r2, 0.f, 0.f, 0.f, 0.f, 0.f};
        beta = pack8<T>(f);
      }
      uint8_t *xa = smem + C::kXOff + q * C::kXBytes;
#pragma unroll 8
      for (int r = 0; r < kBM; ++r) *reinterpret_cast<uint4 *>(xa + x_offset(r, 0)) = beta;
      fence_proxy_async_smem();
    }
    mbar_arrive(&bars->q_full[q]);
    n.q[q] = tile_it + 1;
    return true;
  };
  if (!load_q(0)) return false;
  for (int j = 0; j < t.br.nb; ++j) {
    const int g = kv_base + j;
    const int s = g % C::kStages;
    const uint32_t par = ((g / C::kStages) & 1) ^ 1;
    const int n0 = block_n0<kReverse>(t.br, j);
    if (!wait(&bars->k_empty[s], par)) return false;
    mbar_arrive_expect_tx(&bars->k_full[s], C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_4d(smem + C::kKOff + s * C::kTileBytes + c * C::kChunkBytes, tm_k, &bars->k_full[s], c * 64, t.kvh,
                  n0, t.b);
    n.k = g + 1;
    if (j == 0 && !load_q(1)) return false;
    if (!wait(&bars->v_empty[s], par)) return false;
    mbar_arrive_expect_tx(&bars->v_full[s], C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_4d(smem + C::kVOff + s * C::kTileBytes + c * C::kChunkBytes, tm_v, &bars->v_full[s], c * 64, t.kvh,
                  n0, t.b);
    n.v = g + 1;
    if (bars->abort_flag) return false;
  }
  return true;
}

// Every load issued must have landed before the CTA may exit.  In a normal
// run these phases completed long ago and the waits return at once.
template <int D>
__device__ void tma_drain(Bars *bars, const TmaCounts &n) {
  using C = Cfg<D>;
  for (int q = 0; q < 2; ++q)
    if (n.q[q] > 0) mbar_wait(&bars->q_full[q], (n.q[q] - 1) & 1, kTimeoutNs);
  for (int g = max(0, n.k - C::kStages); g < n.k; ++g)
    mbar_wait(&bars->k_full[g % C::kStages], (g / C::kStages) & 1, kTimeoutNs);
  for (int g = max(0, n.v - C::kStages); g < n.v; ++g)
    mbar_wait(&bars->v_full[g % C::kStages], (g / C::kStages) & 1, kTimeoutNs);
}

// ---------------------------------------------------------------- MMA role
// MMAs of one work item.  kv_base: key blocks of earlier items (ring
// position); blk_base0 / blk_base1: key blocks of earlier items on tile 0 /
// tile 1 (s_full, p_full, o_done complete once per block of their tile);
// tile_it: earlier items (q_full phase).  The last QK^T on each Q buffer is
// followed by a commit to q_empty, so the next item's Q load starts while
// this item finishes.  Tile 1 takes part in all nb blocks; tile 0 (the
// earlier rows) in nb0 of them: the first nb0 in forward order, the last
// nb0 in reverse order (kReverse: the key blocks go last to first, so tile
// 0's blocks, the lowest keys, come at the end).
template <int D, bool kBF16, bool kFold, bool kReverse>
__device__ bool mma_tile(uint8_t *smem, Bars *bars, uint32_t tmem, int nb, int nb0, int tile_it, int kv_base,
                         int blk_base0, int blk_base1) {
  using C = Cfg<D>;
  constexpr uint32_t idesc_qk = idesc_f16(128, kBN, kBF16, false);
  constexpr uint32_t idesc_pv = idesc_f16(128, D, kBF16, true);
  const uint32_t q_base = smem_u32(smem + C::kQOff);
  const uint32_t k_base = smem_u32(smem + C::kKOff);
  const uint32_t v_base = smem_u32(smem + C::kVOff);
  const uint32_t x_base = smem_u32(smem + C::kXOff);
  auto wait = [&](uint64_t *bar, uint32_t par) {
    return mbar_wait_or_abort(bar, par, kTimeoutNs, &bars->abort_flag);
  };

  // Descriptors are built per call from an opaque base plus the step's
  // offset in the 14-bit address field (shared addresses < 256 KB, so the
  // field never carries): the compiler would otherwise keep every stage's
  // descriptors live in registers across the whole loop.
  // S_t = Q_t K^T over D in steps of 16 (32 bytes inside a 128-byte chunk).
  auto issue_qk = [&](int t, int s) {
    const uint32_t d_tmem = tmem + (t ? C::kTmemS1 : C::kTmemS0);
    uint64_t da = smem_desc_sw128(q_base + t * C::kTileBytes, 16, 1024);
    uint64_t db = smem_desc_sw128(k_base + s * C::kTileBytes, 16, 1024);
    asm volatile("" : "+l"(da), "+l"(db));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint64_t off = (uint64_t)(((kk / 4) * C::kChunkBytes + (kk % 4) * 32) >> 4);
      mma_ss(d_tmem, da + off, db + off, idesc_qk, kk > 0 ? 1u : 0u);
    }
    if constexpr (kFold) {
      // S_t += A'_t B'^T: + beta * c for key column c (the ALiBi slope over sm_scale).
      uint64_t dx = smem_desc_noswz(x_base + t * C::kXBytes, 128, 256);
      uint64_t dk = smem_desc_noswz(x_base + 2 * C::kXBytes, 128, 256);
      asm volatile("" : "+l"(dx), "+l"(dk));
      mma_ss(d_tmem, dx, dk, idesc_qk, 1u);
    }
  };
  // O_t (+)= P_t V over the 128 keys in steps of 16 (P: 8 TMEM columns per
  // step; V: 16 rows of 128 bytes per step, MN-major, 64-column chunks 16 KB apart).
  auto issue_pv = [&](int t, int s, bool acc) {
    const uint32_t d_tmem = tmem + (t ? C::kTmemO1 : C::kTmemO0);
    const uint32_t p_tmem = tmem + (t ? C::kTmemS1 : C::kTmemS0);
    uint64_t db = smem_desc_sw128(v_base + s * C::kTileBytes, C::kChunkBytes, 1024);
    asm volatile("" : "+l"(db));
#pragma unroll
    for (int kk = 0; kk < kBN / 16; ++kk)
      mma_ts(d_tmem, p_tmem + kk * 8, db + (uint64_t)((kk * 16 * 128) >> 4), idesc_pv, (acc || kk > 0) ? 1u : 0u);
  };

  // Tile 0 works on blocks j in [lo0, hi0) of the item's sequence.
  const int lo0 = kReverse ? nb - nb0 : 0, hi0 = kReverse ? nb : nb0;
  const uint32_t qpar = tile_it & 1;
  const int s0 = kv_base % C::kStages;
  if (!wait(&bars->k_full[s0], (kv_base / C::kStages) & 1)) return false;
  if (lo0 == 0) {
    if (!wait(&bars->q_full[0], qpar)) return false;
    tc_fence_after();
    issue_qk(0, s0);
    tc_commit(&bars->s_full[0]);
    if (hi0 == 1) tc_commit(&bars->q_empty[0]);
  }
  if (!wait(&bars->q_full[1], qpar)) return false;
  tc_fence_after();
  issue_qk(1, s0);
  tc_commit(&bars->s_full[1]);
  tc_commit(&bars->k_empty[s0]);
  if (nb == 1) tc_commit(&bars->q_empty[1]);
  for (int j = 0; j < nb; ++j) {
    const int g = kv_base + j;
    const int sv = g % C::kStages;
    const int sk = (g + 1) % C::kStages;
    const bool more = j + 1 < nb;
    if (!wait(&bars->v_full[sv], (g / C::kStages) & 1)) return false;
    if (j >= lo0 && j < hi0) {
      if (!wait(&bars->p_full[0], (blk_base0 + j - lo0) & 1)) return false;
      tc_fence_after();
      issue_pv(0, sv, j > lo0);
      tc_commit(&bars->o_done[0]);
    }
    if (more && !wait(&bars->k_full[sk], ((g + 1) / C::kStages) & 1)) return false;
    if (j + 1 >= lo0 && j + 1 < hi0) {
      // Tile 0's first block in reverse order: its Q load is awaited here.
      if (j + 1 == lo0 && !wait(&bars->q_full[0], qpar)) return false;
      tc_fence_after();
      issue_qk(0, sk);
      tc_commit(&bars->s_full[0]);
      if (j + 2 == hi0) tc_commit(&bars->q_empty[0]);
    }
    if (!wait(&bars->p_full[1], (blk_base1 + j) & 1)) return false;
    tc_fence_after();
    issue_pv(1, sv, j > 0);
    tc_commit(&bars->o_done[1]);
    tc_commit(&bars->v_empty[sv]);
    if (more) {
      issue_qk(1, sk);
      tc_commit(&bars->s_full[1]);
      tc_commit(&bars->k_empty[sk]);
      if (j + 2 == nb) tc_commit(&bars->q_empty[1]);
    }
    if (bars->abort_flag) return false;
  }
  return true;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Score of column c (0..127 inside the block) in log2 units, before masking.
template <bool kAlibi, bool kSoftcap>
__device__ __forceinline__ float score2(uint32_t raw, int c, float scale2, float slope2, float jf, float cap_in,
                                        float cap_out) {
  const float v = __uint_as_float(raw);
  float y = kSoftcap ? tanhf(v * cap_in) * cap_out : v * scale2;
  if (kAlibi) y = fmaf(slope2, (float)c, fmaf(slope2, jf, y));
  return y;
}

// Three-input max (sm_100 max.f32 with three sources).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Columns of 32 raw scores (c0..c0+31) outside the row's visible interval
// [lo, hi) become -inf, in place: one bit test and one select per column.
// Used when the score transform maps -inf to -inf (no soft-cap), so the max
// and exponent passes then run unmasked (2^-inf = 0).
__device__ __forceinline__ void mask_chunk(uint32_t (&v)[32], int c0, int lo, int hi) {
  const int a = min(max(lo - c0, 0), 32), e = min(max(hi - c0, 0), 32);
  const uint32_t below_e = e >= 32 ? 0xffffffffu : ((1u << e) - 1u);
  const uint32_t below_a = a >= 32 ? 0xffffffffu : ((1u << a) - 1u);
  const uint32_t vis = below_e & ~below_a;
#pragma unroll
  for (int c = 0; c < 32; ++c) v[c] = (vis & (1u << c)) ? v[c] : 0xff800000u;
}

// Max of 32 scores (columns c0..c0+31), four independent chains.
template <bool kAlibi, bool kSoftcap, bool kMask>
__device__ __forceinline__ float chunk_max(const uint32_t (&v)[32], int c0, int lo, int hi, float scale2,
                                           float slope2, float jf, float cap_in, float cap_out) {
  float m[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) m[i] = -CUDART_INF_F;
  if constexpr (!kAlibi) {
    // Without ALiBi the score transform is increasing (scale2 > 0, tanh), so
    // the row max is the transform of the raw max: one max per column.
#pragma unroll
    for (int c = 0; c < 32; c += 2) {
      float y0 = __uint_as_float(v[c]), y1 = __uint_as_float(v[c + 1]);
      if (kMask) {
        y0 = (c0 + c >= lo && c0 + c < hi) ? y0 : -CUDART_INF_F;
        y1 = (c0 + c + 1 >= lo && c0 + c + 1 < hi) ? y1 : -CUDART_INF_F;
      }
      m[(c >> 1) & 3] = fmax3(m[(c >> 1) & 3], y0, y1);
    }
    const float raw = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
    return raw == -CUDART_INF_F ? raw : score2<false, kSoftcap>(__float_as_uint(raw), 0, scale2, 0.f, 0.f, cap_in, cap_out);
  } else {
#pragma unroll
    for (int c = 0; c < 32; c += 2) {
      float y0 = score2<kAlibi, kSoftcap>(v[c], c0 + c, scale2, slope2, jf, cap_in, cap_out);
      float y1 = score2<kAlibi, kSoftcap>(v[c + 1], c0 + c + 1, scale2, slope2, jf, cap_in, cap_out);
      if (kMask) {
        y0 = (c0 + c >= lo && c0 + c < hi) ? y0 : -CUDART_INF_F;
        y1 = (c0 + c + 1 >= lo && c0 + c + 1 < hi) ? y1 : -CUDART_INF_F;
      }
      m[(c >> 1) & 3] = fmax3(m[(c >> 1) & 3], y0, y1);
    }
    return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
  }
}

// p = 2^(score - m) for 32 columns, packed in pairs into pk[0..15];
// returns the sum of the unrounded p (four independent chains).
template <typename T, bool kAlibi, bool kSoftcap, bool kMask>
__device__ __forceinline__ float chunk_exp(const uint32_t (&v)[32], uint32_t (&pk)[16], int c0, int lo, int hi,
                                           float scale2, float slope2, float jf, float cap_in, float cap_out,
                                           float m) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    float y0 = score2<kAlibi, kSoftcap>(v[c], c0 + c, scale2, slope2, jf, cap_in, cap_out);
    float y1 = score2<kAlibi, kSoftcap>(v[c + 1], c0 + c + 1, scale2, slope2, jf, cap_in, cap_out);
    if (kMask) {
      y0 = (c0 + c >= lo && c0 + c < hi) ? y0 : -CUDART_INF_F;
      y1 = (c0 + c + 1 >= lo && c0 + c + 1 < hi) ? y1 : -CUDART_INF_F;
    }
    const float p0 = ex2_approx(y0 - m), p1 = ex2_approx(y1 - m);
    s[(c >> 1) & 3] += p0 + p1;
    pk[c / 2] = pack2<T>(p0, p1);
  }
  return (s[0] + s[1]) + (s[2] + s[3]);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): two lanes of work per
// instruction for the scale-and-subtract and the running sum of the plain
// (and folded-ALiBi) exponent pass.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// p = 2^(v * scale2 - m) for 32 raw scores (masked ones already -inf),
// packed in pairs into pk[0..15]; returns the sum of the unrounded p.
template <typename T>
__device__ __forceinline__ float chunk_exp_plain2(const uint32_t (&v)[32], uint32_t (&pk)[16], float scale2, float m) {
  uint64_t acc0 = f2(0.f, 0.f), acc1 = f2(0.f, 0.f);
  const uint64_t sc = f2(scale2, scale2), nm = f2(-m, -m);
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    float y0, y1;
    f2_split(fma2(f2(__uint_as_float(v[c]), __uint_as_float(v[c + 1])), sc, nm), y0, y1);
    const float p0 = ex2_approx(y0), p1 = ex2_approx(y1);
    if ((c >> 1) & 1)
      acc1 = add2(acc1, f2(p0, p1));
    else
      acc0 = add2(acc0, f2(p0, p1));
    pk[c / 2] = pack2<T>(p0, p1);
  }
  float a, b, cc, d;
  f2_split(acc0, a, b);
  f2_split(acc1, cc, d);
  return (a + b) + (cc + d);
}

// One KV block of one row: load S (128 columns, one TMEM round trip), row
// max, the rescale decision, P = 2^(s - m) written back over S as 16-bit
// pairs, and the running sum.  kMask selects the per-column interval test;
// the two variants are separate code paths.
template <typename T, bool kAlibi, bool kSoftcap, bool kMask>
__device__ __forceinline__ void softmax_block(uint32_t tS, int n0, int kv_offset, int lo, int hi, float scale2,
                                              float slope2,
                                              float cap_in, float cap_out, float &m_used, float &l, float &alpha,
                                              bool &rescale) {
  const float kNegInf = -CUDART_INF_F;
  const float jf = (float)(n0 + kv_offset);
  // An opaque per-block copy of the slope keeps the compiler from hoisting
  // 128 per-column products slope * c out of the block loop into registers.
  float sl = slope2;
  asm volatile("" : "+f"(sl));
  // ALiBi without soft-cap is folded into S (the per-column part beta * c,
  // see x_offset); what is left is one constant per block, added to the max
  // and taken out of the exponent's offset.  kCol: per-column bias here.
  constexpr bool kFold = kAlibi && !kSoftcap;
  constexpr bool kCol = kAlibi && !kFold;
  const float off = kFold ? sl * jf : 0.f;
  uint32_t sr[4][32];
#pragma unroll
  for (int q = 0; q < 4; ++q) tmem_ld32(tS + q * 32, sr[q]);
  tmem_wait_ld();
#pragma unroll
  for (int q = 0; q < 4; ++q) reg_fence32(sr[q]);
  // Without soft-cap the mask is applied once, to the raw scores; with it,
  // after the transform in both passes (tanh(-inf) is not -inf).
  constexpr bool kMaskRaw = kMask && !kSoftcap;
  constexpr bool kMaskPass = kMask && kSoftcap;
  if constexpr (kMaskRaw) {
#pragma unroll
    for (int q = 0; q < 4; ++q) mask_chunk(sr[q], q * 32, lo, hi);
  }
  float mx = kNegInf;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    mx = fmaxf(mx, chunk_max<kCol, kSoftcap, kMaskPass>(sr[q], q * 32, lo, hi, scale2, sl, jf, cap_in, cap_out));
  if constexpr (kFold) mx += off;  // -inf stays -inf
  // Fresh names for the raw scores: pass 2 recomputes each transformed
  // score instead of keeping pass 1's values alive next to the raw row.
#pragma unroll
  for (int q = 0; q < 4; ++q) reg_fence32(sr[q]);
  const float m_new = fmaxf(m_used, mx);
  if (m_used == kNegInf) {
    m_used = m_new;  // nothing accumulated yet: O and l are zero
  } else if (m_new > m_used + rescale_threshold<T>()) {
    alpha = ex2_approx(m_used - m_new);
    m_used = m_new;
    rescale = true;
  }
  const float m_eff = (m_used == kNegInf) ? 0.f : m_used;
  float psum = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t pk[16];
    if constexpr (!kCol && !kSoftcap)
      psum += chunk_exp_plain2<T>(sr[q], pk, scale2, m_eff - off);
    else
      psum += chunk_exp<T, kCol, kSoftcap, kMaskPass>(sr[q], pk, q * 32, lo, hi, scale2, sl, jf, cap_in, cap_out,
                                                    m_eff - off);
    tmem_st16(tS + q * 16, pk);
  }
  l = l * alpha + psum;
}

// 4 x 4 transpose of 16-byte pieces inside each group of four lanes: on
// entry u[j] is piece j of this lane's row, on exit u[k] is piece (lane % 4)
// of row k of the group.  Two rounds of exchanges with lane ^ 2 and lane ^ 1,
// each swapping the two pieces whose index bit differs from the lane's.
__device__ __forceinline__ void xchg_unit(uint4 &dst, const uint4 &src, int mask) {
  dst.x = __shfl_xor_sync(0xffffffffu, src.x, mask);
  dst.y = __shfl_xor_sync(0xffffffffu, src.y, mask);
  dst.z = __shfl_xor_sync(0xffffffffu, src.z, mask);
  dst.w = __shfl_xor_sync(0xffffffffu, src.w, mask);
}
__device__ __forceinline__ void transpose_units4(uint4 (&u)[4]) {
  const int i = threadIdx.x & 3;
  const bool b1 = (i >> 1) & 1, b0 = i & 1;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint4 send = b1 ? u[k] : u[k | 2];
    uint4 recv;
    xchg_unit(recv, send, 2);
    if (b1)
      u[k] = recv;
    else
      u[k | 2] = recv;
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint4 send = b0 ? u[2 * k] : u[2 * k + 1];
    uint4 recv;
    xchg_unit(recv, send, 1);
    if (b0)
      u[2 * k] = recv;
    else
      u[2 * k + 1] = recv;
  }
}

// ------------------------------------------------------------ softmax role
// One work item.  Thread r of warpgroup t owns query row r of tile t (TMEM
// lane r).  blk_base: key blocks of earlier items (barrier phases).  Returns
// false when the kernel is aborting.
template <typename T, int D, bool kAlibi, bool kSoftcap>
__device__ bool softmax_tile(const AttnArgs &a, Bars *bars, uint32_t tmem, int warp, const Work &w, int blk_base) {
  using C = Cfg<D>;
  const float kNegInf = -CUDART_INF_F;
  const int t = warp / 4;
  BlockRange br = w.br;
  if (t == 0) br.nb = w.nb0;
  const int m0 = w.m0, h = w.h, b = w.b, ql = w.ql, kl = w.kl;
  const int r = threadIdx.x % kBM;
  const int row0 = m0 + t * kBM;
  const int qi = row0 + r;
  const int off = diag_shift(a, ql, kl);
  const int diag = qi + off;
  const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
  const uint32_t tS = tmem + lane_off + (t ? C::kTmemS1 : C::kTmemS0);
  const uint32_t tO = tmem + lane_off + (t ? C::kTmemO1 : C::kTmemO0);
  const float scale2 = a.sm_scale * kLog2e;
  const float slope2 = kAlibi ? a.alibi[h] * kLog2e : 0.f;
  const float cap_in = kSoftcap ? a.sm_scale / a.softcap : 0.f;
  const float cap_out = kSoftcap ? a.softcap * kLog2e : 0.f;
  float m_used = kNegInf, l = 0.f;
  bool aborted = false;

  for (int j = 0; j < br.nb; ++j) {
    const int n0 = block_n0<kAlibi>(br, j);
    bool ok = mbar_wait_or_abort(&bars->s_full[t], (blk_base + j) & 1, kTimeoutNs, &bars->abort_flag);
    if (!__all_sync(0xffffffffu, ok)) {
      set_abort(bars, a.err);
      aborted = true;
      break;
    }
    tc_fence_after();
    // Visible keys of this row inside the block form one interval [lo, hi)
    // (bottom-right causal and length bound cut above, the window below).
    int lo = 0, hi = kBN;
    const bool need_mask = (n0 + kBN > kl) || (a.causal && n0 + kBN - 1 > row0 + off) ||
                           (a.window >= 0 && row0 + kBM - 1 + off - n0 > a.window);
    if (need_mask) {
      hi = min(kBN, kl - n0);
      if (a.causal) hi = min(hi, diag - n0 + 1);
      if (a.window >= 0) lo = max(0, diag - a.window - n0);
    }
    float alpha = 1.f;
    bool rescale = false;
    if (need_mask && __all_sync(0xffffffffu, hi <= lo)) {
      // No row of this warp sees a key of the block: P = 0, m and l unchanged.
      uint32_t z[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) z[c] = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_st16(tS + q * 16, z);
    } else if (need_mask)
      softmax_block<T, kAlibi, kSoftcap, true>(tS, n0, a.kv_offset, lo, hi, scale2, slope2, cap_in, cap_out, m_used, l, alpha,
                                               rescale);
    else
      softmax_block<T, kAlibi, kSoftcap, false>(tS, n0, a.kv_offset, lo, hi, scale2, slope2, cap_in, cap_out, m_used, l, alpha,
                                                rescale);
    if (__any_sync(0xffffffffu, rescale)) {
      // O_t holds blocks 0..j-1 once PV_t(j-1) is done; rescale it in place.
      ok = mbar_wait_or_abort(&bars->o_done[t], (blk_base + j - 1) & 1, kTimeoutNs, &bars->abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        set_abort(bars, a.err);
        aborted = true;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int ch = 0; ch < D / 32; ++ch) {
        uint32_t o[32];
        tmem_ld32(tO + ch * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
        tmem_st32(tO + ch * 32, o);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars->p_full[t]);
  }

  // Epilogue: O_t / l -> global (rows past q_len as zeros), lse.
  if (!aborted && br.nb > 0) {
    bool ok = mbar_wait_or_abort(&bars->o_done[t], (blk_base + br.nb - 1) & 1, kTimeoutNs, &bars->abort_flag);
    if (!__all_sync(0xffffffffu, ok)) {
      set_abort(bars, a.err);
      aborted = true;
    } else {
      tc_fence_after();
    }
  }
  const bool have = !aborted && br.nb > 0;
  const bool valid = qi < ql && l > 0.f;  // padded rows and rows with no visible key -> 0
  const float inv = valid ? 1.f / l : 0.f;
  // Each group of four lanes (four consecutive rows) swaps 16-byte pieces so
  // that every store instruction writes 64 contiguous bytes of 8 rows.
  const int gi = threadIdx.x & 3;
  const int qi_group = qi - gi;
  // Row `row` of this (batch, head) goes to obase + row * orow.  Scattered
  // output (a.xs_n > 0): global row R = xs_row_base + row belongs to
  // destination R / xs_slice, laid out [batch, xs_slice, H, D] there; the
  // four rows of a lane group share one destination (slice and base are
  // multiples of 16).
  T *obase;
  long long orow;
  if (a.xs_n > 0) {
    const int rg = a.xs_row_base + qi_group;
    const int p = rg / a.xs_slice;
    orow = (long long)a.H * a.D;
    obase = static_cast<T *>(a.xs_o[p]) + ((long long)b * a.xs_slice + (rg - p * a.xs_slice) - qi_group) * orow +
            (long long)h * a.D;
  } else {
    orow = a.os[1];
    obase = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
  }
#pragma unroll 1
  for (int ch = 0; ch < D / 32; ++ch) {
    uint32_t o[32];
    if (have) {
      tmem_ld32(tO + ch * 32, o);
      tmem_wait_ld();
      reg_fence32(o);
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = 0u;
    }
    uint32_t w[16];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      w[c] = valid ? pack2<T>(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv) : 0u;
    uint4 u[4];
#pragma unroll
    for (int v4 = 0; v4 < 4; ++v4) u[v4] = make_uint4(w[4 * v4], w[4 * v4 + 1], w[4 * v4 + 2], w[4 * v4 + 3]);
    transpose_units4(u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int row = qi_group + k;
      if (row < a.Sq) *reinterpret_cast<uint4 *>(obase + (long long)row * orow + ch * 32 + gi * 8) = u[k];
    }
  }
  // The unit's last item also writes the rows past the query length that no
  // item covers (items starting past it are skipped): zeros, lse -inf.
  if (a.xs_n == 0 && m0 + kTiles * kBM >= ql && m0 + kTiles * kBM < a.Sq) {
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    T *const zbase = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
    for (int row = m0 + kTiles * kBM + t * kBM + r; row < a.Sq; row += kTiles * kBM) {
#pragma unroll 4
      for (int c = 0; c < D; c += 8) *reinterpret_cast<uint4 *>(zbase + (long long)row * a.os[1] + c) = z;
      if (a.lse != nullptr) a.lse[((long long)b * a.H + h) * a.Sq + row] = kNegInf;
    }
  }
  const float lse_v = valid ? (m_used + log2f(l)) * kLn2 : kNegInf;
  if (a.xs_n > 0) {
    if (qi < a.Sq) {
      const int rr = a.xs_row_base + qi;
      const int p = rr / a.xs_slice;
      a.xs_lse[p][((long long)b * a.H + h) * a.xs_slice + (rr - p * a.xs_slice)] = lse_v;
    }
  } else if (a.lse != nullptr && qi < a.Sq) {
    a.lse[((long long)b * a.H + h) * a.Sq + qi] = lse_v;
  }
  return !aborted;
}

// ------------------------------------------------------------------ kernel
// With a work counter the grid has one CTA per SM and each CTA runs work
// items back to back, so barrier set-up and tensor-memory allocation happen
// once per CTA, and the next item's Q / K / V loads and first QK^T overlap
// the current item's last block and epilogue.  Without one, one CTA per item.
template <typename T, int D, bool kAlibi, bool kSoftcap>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_sm100_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const AttnArgs a, const int n_mblocks,
                      const int group_units, const int n_work, int *work_ctr) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled tiles want 1024-byte aligned shared-memory addresses.
  // Offsetting smem_raw (rather than rounding a cast integer) keeps every
  // derived pointer known to be in shared memory, so barrier and flag
  // addresses stay 32-bit shared-window values instead of generic pointers
  // the compiler would spill.
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Bars *bars = reinterpret_cast<Bars *>(smem + C::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int q = 0; q < kTiles; ++q) {
      mbar_init(&bars->q_full[q], 1);
      mbar_init(&bars->q_empty[q], 1);
    }
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], kBM);
      mbar_init(&bars->o_done[t], 1);
    }
    for (int i = 0; i < kSchedSlots; ++i) {
      mbar_init(&bars->sched_full[i], 1);
      mbar_init(&bars->sched_empty[i], kSchedConsumers);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  constexpr bool kFold = kAlibi && !kSoftcap;
  if constexpr (kFold) {
    // B' row c = [c, c, c, 0, ...] in columns 0-15; A'_0 and A'_1 zero (their
    // columns 0-2 are written per work item).  256 16-byte units per operand.
    for (int u = threadIdx.x; u < 3 * 256; u += kThreads) {
      const int op = u >> 8, e = u & 255;
      const int r = (e >> 4) * 8 + (e & 7), khalf = (e >> 3) & 1;
      const float c = (op == 2 && khalf == 0) ? (float)r : 0.f;
      const float f[8] = {c, c, c, 0.f, 0.f, 0.f, 0.f, 0.f};
      *reinterpret_cast<uint4 *>(smem + C::kXOff + op * C::kXBytes + x_offset(r, khalf * 8)) = pack8<T>(f);
    }
    fence_proxy_async_smem();
  }
  if (warp == kTmaWarp && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&bars->tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp >= 8) {
    regs_decrease<kRegsControl>();
    if (warp == kTmaWarp && lane == 0) {
      TmaCounts n;
      int kv = 0, it = 0;
      int w = (int)blockIdx.x;
      for (int seq = 0;;) {
        Work t{};
        if (w < n_work) {
          t = decode_work(a, w, n_mblocks, group_units);
          // Rows past the sequence's query length: nothing to compute, and the
          // unit's last item zero-fills them (softmax_tile), so the item is
          // not published at all.
          if (t.m0 >= t.ql && t.m0 > 0) {
            w = work_ctr != nullptr ? (int)gridDim.x + atomicAdd(work_ctr, 1) : n_work;
            continue;
          }
        }
        if (!sched_publish_item(bars, seq++, w, t)) {
          set_abort(bars, a.err);
          break;
        }
        if (w >= n_work) break;
        if (t.br.nb > 0) {
          const bool ok = tma_tile<T, D, kFold, kAlibi>(&tm_q, &tm_k, &tm_v, smem, bars, t, it, kv, n, a);
          kv += t.br.nb;
          ++it;
          if (!ok) {
            set_abort(bars, a.err);
            break;
          }
        }
        w = work_ctr != nullptr ? (int)gridDim.x + atomicAdd(work_ctr, 1) : n_work;
      }
      tma_drain<D>(bars, n);
    } else if (warp == kMmaWarp && lane == 0) {
      int kv = 0, it = 0, blk0 = 0;
      for (int seq = 0;; ++seq) {
        Work t;
        const int w = sched_take_item(bars, seq, false, t);
        if (w < 0) {
          set_abort(bars, a.err);
          break;
        }
        if (w >= n_work) break;
        if (t.br.nb == 0) continue;
        const bool ok = mma_tile<D, std::is_same<T, __nv_bfloat16>::value, kFold, kAlibi>(smem, bars, tmem, t.br.nb,
                                                                                            t.nb0, it, kv, blk0, kv);
        kv += t.br.nb;
        blk0 += t.nb0;
        ++it;
        if (!ok) {
          set_abort(bars, a.err);
          break;
        }
      }
      // Drain: all MMAs this thread issued complete before tensor memory is freed.
      tc_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, kTimeoutNs);
    }
  } else {
    regs_increase<kRegsSoftmax>();
    int blk = 0;
    for (int seq = 0;; ++seq) {
      Work t;
      const int w = sched_take_item(bars, seq, true, t);
      if (w < 0) {
        set_abort(bars, a.err);
        break;
      }
      if (w >= n_work) break;
      if (!softmax_tile<T, D, kAlibi, kSoftcap>(a, bars, tmem, warp, t, blk)) break;
      blk += warp < 4 ? t.nb0 : t.br.nb;
    }
    // Scattered output may be other GPUs' memory: make this thread's writes
    // visible system-wide once, after its last item, before the kernel ends.
    if (a.xs_n > 0) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ========================================================== head_dim 256
// One 128-row query tile per work item.  Tensor memory: two S buffers
// (S_0, S_1: 128 fp32 columns each) and O (256 columns).  The MMA thread
// keeps QK^T one key block ahead of PV -- QK(0), QK(1), PV(0), QK(2), PV(1),
// ... -- so the tensor core computes the next scores and the previous PV
// while the softmax warpgroup works on the current block (at head_dim 256
// that is ~2960 tensor cycles per block against ~2100 cycles of softmax).
// Shared memory holds Q and one 64 KB slot each for K and V (plus the ALiBi
// operands); K and V have their own TMA threads, so a K load never queues
// behind a V load.
struct Cfg256 {
  static constexpr int D = 256;
  static constexpr int kChunks = D / 64;
  static constexpr int kChunkBytes = 128 * 128;
  static constexpr int kTileBytes = 128 * D * 2;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kTileBytes;
  static constexpr int kVOff = 2 * kTileBytes;
  static constexpr int kXOff = 3 * kTileBytes;  // A' (8 KB) then B' (8 KB)
  static constexpr int kXBytes = 8192;
  static constexpr int kBarOff = kXOff + 2 * kXBytes;
  static constexpr int kSmemBytes = kBarOff + 1024 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
  static constexpr uint32_t kTmemS0 = 0, kTmemS1 = 128, kTmemO = 256, kTmemCols = 512;
};
constexpr int kThreads256 = 256;  // warps 0-3 softmax, 4 MMA, 5 K + Q loads, 6 V loads, 7 idle
constexpr int kMmaWarp256 = 4, kKWarp256 = 5, kVWarp256 = 6;
constexpr int kSchedConsumers256 = 1 + 1 + 4;  // MMA thread, V thread, one lane per softmax warp

struct Bars256 {
  uint64_t q_full, q_empty, k_full, k_empty, v_full, v_empty;
  uint64_t s_full[2], p_full[2], o_done;
  uint64_t drain;
  uint64_t sched_full[kSchedSlots], sched_empty[kSchedSlots];
  int sched_w[kSchedSlots];
  uint32_t tmem_base;
  volatile int abort_flag;
};
static_assert(sizeof(Bars256) <= 1024, "barrier region");

// K / Q loads of one item (the K thread); g0: key blocks of earlier items.
template <bool kFold, bool kReverse>
__device__ bool tma_k256(const CUtensorMap *tm_q, const CUtensorMap *tm_k, uint8_t *smem, Bars256 *bars,
                         const Work &t, int tile_it, int g0, int &k_issued, int &q_issued, uint4 beta) {
  using C = Cfg256;
  auto wait = [&](uint64_t *bar, uint32_t par) {
    return mbar_wait_or_abort(bar, par, kTimeoutNs, &bars->abort_flag);
  };
  if (tile_it > 0 && !wait(&bars->q_empty, (tile_it - 1) & 1)) return false;
  if constexpr (kFold) {
    uint8_t *xa = smem + C::kXOff;
#pragma unroll 8
    for (int r = 0; r < kBM; ++r) *reinterpret_cast<uint4 *>(xa + x_offset(r, 0)) = beta;
    fence_proxy_async_smem();
  }
  mbar_arrive_expect_tx(&bars->q_full, C::kTileBytes);
  for (int c = 0; c < C::kChunks; ++c)
    tma_load_4d(smem + C::kQOff + c * C::kChunkBytes, tm_q, &bars->q_full, c * 64, t.h, t.m0, t.b);
  q_issued = tile_it + 1;
  for (int j = 0; j < t.br.nb; ++j) {
    const int g = g0 + j;
    if (!wait(&bars->k_empty, (g & 1) ^ 1)) return false;
    mbar_arrive_expect_tx(&bars->k_full, C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_4d(smem + C::kKOff + c * C::kChunkBytes, tm_k, &bars->k_full, c * 64, t.kvh,
                  block_n0<kReverse>(t.br, j), t.b);
    k_issued = g + 1;
    if (bars->abort_flag) return false;
  }
  return true;
}

// V loads of one item (the V thread).
template <bool kReverse>
__device__ bool tma_v256(const CUtensorMap *tm_v, uint8_t *smem, Bars256 *bars, const Work &t, int g0,
                         int &v_issued) {
  using C = Cfg256;
  for (int j = 0; j < t.br.nb; ++j) {
    const int g = g0 + j;
    if (!mbar_wait_or_abort(&bars->v_empty, (g & 1) ^ 1, kTimeoutNs, &bars->abort_flag)) return false;
    mbar_arrive_expect_tx(&bars->v_full, C::kTileBytes);
    for (int c = 0; c < C::kChunks; ++c)
      tma_load_4d(smem + C::kVOff + c * C::kChunkBytes, tm_v, &bars->v_full, c * 64, t.kvh,
                  block_n0<kReverse>(t.br, j), t.b);
    v_issued = g + 1;
    if (bars->abort_flag) return false;
  }
  return true;
}

// MMAs of one item: QK(g0), QK(g0 + 1), then per block PV(g), QK(g + 2).
// Block g's scores live in S_(g & 1); s_full / p_full of a buffer complete
// once per block that uses it (phase g >> 1); o_done once per block.
template <bool kBF16, bool kFold>
__device__ bool mma_256(uint8_t *smem, Bars256 *bars, uint32_t tmem, int nb, int tile_it, int g0) {
  using C = Cfg256;
  constexpr int D = C::D;
  constexpr uint32_t idesc_qk = idesc_f16(128, kBN, kBF16, false);
  constexpr uint32_t idesc_pv = idesc_f16(128, D, kBF16, true);
  const uint32_t q_base = smem_u32(smem + C::kQOff);
  const uint32_t k_base = smem_u32(smem + C::kKOff);
  const uint32_t v_base = smem_u32(smem + C::kVOff);
  const uint32_t x_base = smem_u32(smem + C::kXOff);
  auto wait = [&](uint64_t *bar, uint32_t par) {
    return mbar_wait_or_abort(bar, par, kTimeoutNs, &bars->abort_flag);
  };
  auto issue_qk = [&](int buf) {
    const uint32_t d_tmem = tmem + (buf ? C::kTmemS1 : C::kTmemS0);
    uint64_t da = smem_desc_sw128(q_base, 16, 1024);
    uint64_t db = smem_desc_sw128(k_base, 16, 1024);
    asm volatile("" : "+l"(da), "+l"(db));
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint64_t off = (uint64_t)(((kk / 4) * C::kChunkBytes + (kk % 4) * 32) >> 4);
      mma_ss(d_tmem, da + off, db + off, idesc_qk, kk > 0 ? 1u : 0u);
    }
    if constexpr (kFold) {
      uint64_t dx = smem_desc_noswz(x_base, 128, 256);
      uint64_t dk = smem_desc_noswz(x_base + C::kXBytes, 128, 256);
      asm volatile("" : "+l"(dx), "+l"(dk));
      mma_ss(d_tmem, dx, dk, idesc_qk, 1u);
    }
  };
  auto issue_pv = [&](int buf, bool acc) {
    const uint32_t d_tmem = tmem + C::kTmemO;
    const uint32_t p_tmem = tmem + (buf ? C::kTmemS1 : C::kTmemS0);
    uint64_t db = smem_desc_sw128(v_base, C::kChunkBytes, 1024);
    asm volatile("" : "+l"(db));
#pragma unroll
    for (int kk = 0; kk < kBN / 16; ++kk)
      mma_ts(d_tmem, p_tmem + kk * 8, db + (uint64_t)((kk * 16 * 128) >> 4), idesc_pv, (acc || kk > 0) ? 1u : 0u);
  };
  // QK^T of block g (its K is in the single K slot).
  auto qk_block = [&](int g, bool last) {
    if (!wait(&bars->k_full, g & 1)) return false;
    tc_fence_after();
    issue_qk(g & 1);
    tc_commit(&bars->s_full[g & 1]);
    tc_commit(&bars->k_empty);
    if (last) tc_commit(&bars->q_empty);
    return true;
  };
  if (!wait(&bars->q_full, tile_it & 1)) return false;
  if (!qk_block(g0, nb == 1)) return false;
  if (nb > 1 && !qk_block(g0 + 1, nb == 2)) return false;
  for (int j = 0; j < nb; ++j) {
    const int g = g0 + j;
    if (!wait(&bars->v_full, g & 1) || !wait(&bars->p_full[g & 1], (g >> 1) & 1)) return false;
    tc_fence_after();
    issue_pv(g & 1, j > 0);
    tc_commit(&bars->o_done);
    tc_commit(&bars->v_empty);
    if (j + 2 < nb && !qk_block(g + 2, j + 3 == nb)) return false;
    if (bars->abort_flag) return false;
  }
  return true;
}

// Softmax of one item (warps 0-3, thread r = row r = TMEM lane r), then the
// epilogue.  g0: key blocks of earlier items.
template <typename T, bool kAlibi, bool kSoftcap>
__device__ bool softmax_256(const AttnArgs &a, Bars256 *bars, uint32_t tmem, int warp, const Work &w, int g0) {
  using C = Cfg256;
  constexpr int D = C::D;
  const float kNegInf = -CUDART_INF_F;
  const BlockRange br = w.br;
  const int m0 = w.m0, h = w.h, b = w.b, ql = w.ql, kl = w.kl;
  const int r = threadIdx.x;  // warps 0-3
  const int qi = m0 + r;
  const int off = diag_shift(a, ql, kl);
  const int diag = qi + off;
  const uint32_t lane_off = (uint32_t)((warp % 4) * 32) << 16;
  const uint32_t tO = tmem + lane_off + C::kTmemO;
  const float scale2 = a.sm_scale * kLog2e;
  const float slope2 = kAlibi ? a.alibi[h] * kLog2e : 0.f;
  const float cap_in = kSoftcap ? a.sm_scale / a.softcap : 0.f;
  const float cap_out = kSoftcap ? a.softcap * kLog2e : 0.f;
  float m_used = kNegInf, l = 0.f;
  bool aborted = false;

  for (int j = 0; j < br.nb; ++j) {
    const int g = g0 + j;
    const int n0 = block_n0<kAlibi>(br, j);
    const uint32_t tS = tmem + lane_off + ((g & 1) ? C::kTmemS1 : C::kTmemS0);
    bool ok = mbar_wait_or_abort(&bars->s_full[g & 1], (g >> 1) & 1, kTimeoutNs, &bars->abort_flag);
    if (!__all_sync(0xffffffffu, ok)) {
      set_abort(bars, a.err);
      aborted = true;
      break;
    }
    tc_fence_after();
    int lo = 0, hi = kBN;
    const bool need_mask = (n0 + kBN > kl) || (a.causal && n0 + kBN - 1 > m0 + off) ||
                           (a.window >= 0 && m0 + kBM - 1 + off - n0 > a.window);
    if (need_mask) {
      hi = min(kBN, kl - n0);
      if (a.causal) hi = min(hi, diag - n0 + 1);
      if (a.window >= 0) lo = max(0, diag - a.window - n0);
    }
    float alpha = 1.f;
    bool rescale = false;
    if (need_mask && __all_sync(0xffffffffu, hi <= lo)) {
      uint32_t z[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) z[c] = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_st16(tS + q * 16, z);
    } else if (need_mask) {
      softmax_block<T, kAlibi, kSoftcap, true>(tS, n0, a.kv_offset, lo, hi, scale2, slope2, cap_in, cap_out, m_used,
                                               l, alpha, rescale);
    } else {
      softmax_block<T, kAlibi, kSoftcap, false>(tS, n0, a.kv_offset, lo, hi, scale2, slope2, cap_in, cap_out, m_used,
                                                l, alpha, rescale);
    }
    if (__any_sync(0xffffffffu, rescale)) {
      // O holds blocks 0..j-1 once PV(g - 1) is done; rescale it in place.
      // (S(g) arriving means PV(g - 2) completed, so o_done is at most one
      // phase behind the one waited for.)
      ok = mbar_wait_or_abort(&bars->o_done, (g - 1) & 1, kTimeoutNs, &bars->abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        set_abort(bars, a.err);
        aborted = true;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int ch = 0; ch < D / 32; ++ch) {
        uint32_t o[32];
        tmem_ld32(tO + ch * 32, o);
        tmem_wait_ld();
        reg_fence32(o);
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
        tmem_st32(tO + ch * 32, o);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars->p_full[g & 1]);
  }

  if (!aborted && br.nb > 0) {
    // QK(g) is issued before PV(g - 1), so when the last block's scores
    // arrived only PV(last - 2) was known complete: wait for o_done's phase
    // last - 1 and then last (a parity wait must never be two phases ahead
    // of the barrier, or it would match the older phase of equal parity).
    const int gl = g0 + br.nb - 1;
    bool ok = true;
    if (br.nb >= 2) ok = mbar_wait_or_abort(&bars->o_done, (gl - 1) & 1, kTimeoutNs, &bars->abort_flag);
    ok = ok && mbar_wait_or_abort(&bars->o_done, gl & 1, kTimeoutNs, &bars->abort_flag);
    if (!__all_sync(0xffffffffu, ok)) {
      set_abort(bars, a.err);
      aborted = true;
    } else {
      tc_fence_after();
    }
  }
  const bool have = !aborted && br.nb > 0;
  const bool valid = qi < ql && l > 0.f;
  const float inv = valid ? 1.f / l : 0.f;
  const int gi = threadIdx.x & 3;
  const int qi_group = qi - gi;
  T *const obase = static_cast<T *>(a.o) + b * a.os[0] + h * a.os[2];
  // Two 32-column chunks of O per tensor-memory wait (one wait per 64
  // columns halves the load latency the 256-column epilogue waits out).
#pragma unroll 1
  for (int ch2 = 0; ch2 < D / 32; ch2 += 2) {
    uint32_t o2[2][32];
    if (have) {
      tmem_ld32(tO + ch2 * 32, o2[0]);
      tmem_ld32(tO + (ch2 + 1) * 32, o2[1]);
      tmem_wait_ld();
      reg_fence32(o2[0]);
      reg_fence32(o2[1]);
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) o2[0][c] = o2[1][c] = 0u;
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
    const int ch = ch2 + half;
    uint32_t (&o)[32] = o2[half];
    uint32_t wv[16];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      wv[c] = valid ? pack2<T>(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv) : 0u;
    uint4 u[4];
#pragma unroll
    for (int v4 = 0; v4 < 4; ++v4) u[v4] = make_uint4(wv[4 * v4], wv[4 * v4 + 1], wv[4 * v4 + 2], wv[4 * v4 + 3]);
    transpose_units4(u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int row = qi_group + k;
      if (row < a.Sq) *reinterpret_cast<uint4 *>(obase + (long long)row * a.os[1] + ch * 32 + gi * 8) = u[k];
    }
    }
  }
  if (a.lse != nullptr && qi < a.Sq)
    a.lse[((long long)b * a.H + h) * a.Sq + qi] = valid ? (m_used + log2f(l)) * kLn2 : kNegInf;
  return !aborted;
}

template <typename T, bool kAlibi, bool kSoftcap>
__global__ void __launch_bounds__(kThreads256, 1)
    fmha_sm100_d256_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const AttnArgs a, const int n_mblocks,
                           const int group_units, const int n_work, int *work_ctr) {
  using C = Cfg256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Bars256 *bars = reinterpret_cast<Bars256 *>(smem + C::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr bool kFold = kAlibi && !kSoftcap;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    mbar_init(&bars->k_full, 1);
    mbar_init(&bars->k_empty, 1);
    mbar_init(&bars->v_full, 1);
    mbar_init(&bars->v_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], kBM);
    }
    mbar_init(&bars->o_done, 1);
    for (int i = 0; i < kSchedSlots; ++i) {
      mbar_init(&bars->sched_full[i], 1);
      mbar_init(&bars->sched_empty[i], kSchedConsumers256);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (kFold) {
    // B' row c = [c, c, c, 0, ...]; A' zero (its columns 0-2 are written per item).
    for (int u = threadIdx.x; u < 2 * 256; u += kThreads256) {
      const int op = u >> 8, e = u & 255;
      const int r = (e >> 4) * 8 + (e & 7), khalf = (e >> 3) & 1;
      const float c = (op == 1 && khalf == 0) ? (float)r : 0.f;
      const float f[8] = {c, c, c, 0.f, 0.f, 0.f, 0.f, 0.f};
      *reinterpret_cast<uint4 *>(smem + C::kXOff + op * C::kXBytes + x_offset(r, khalf * 8)) = pack8<T>(f);
    }
    fence_proxy_async_smem();
  }
  if (warp == kKWarp256 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  if (warp == kMmaWarp256) {
    tmem_alloc(&bars->tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kKWarp256 && lane == 0) {
    int g = 0, it = 0, k_issued = 0, q_issued = 0;
    int w = (int)blockIdx.x;
    for (int seq = 0;; ++seq) {
      if (!sched_publish(bars, seq, w)) {
        set_abort(bars, a.err);
        break;
      }
      if (w >= n_work) break;
      const Work t = decode_work(a, w, n_mblocks, group_units, kBM);
      if (t.br.nb > 0) {
        uint4 beta = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (kFold) {
          const float bb = a.alibi[t.h] / a.sm_scale;
          const float r1 = bb - Elem<T>::to_f(Elem<T>::from_f(bb));
          const float r2 = r1 - Elem<T>::to_f(Elem<T>::from_f(r1));
          const float f[8] = {bb, r1, r2, 0.f, 0.f, 0.f, 0.f, 0.f};
          beta = pack8<T>(f);
        }
        const bool ok = tma_k256<kFold, kAlibi>(&tm_q, &tm_k, smem, bars, t, it, g, k_issued, q_issued, beta);
        g += t.br.nb;
        ++it;
        if (!ok) {
          set_abort(bars, a.err);
          break;
        }
      }
      w = work_ctr != nullptr ? (int)gridDim.x + atomicAdd(work_ctr, 1) : n_work;
    }
    // Drain: every issued load lands before the CTA exits.
    if (q_issued > 0) mbar_wait(&bars->q_full, (q_issued - 1) & 1, kTimeoutNs);
    if (k_issued > 0) mbar_wait(&bars->k_full, (k_issued - 1) & 1, kTimeoutNs);
  } else if (warp == kVWarp256 && lane == 0) {
    int g = 0, v_issued = 0;
    for (int seq = 0;; ++seq) {
      const int w = sched_take(bars, seq, false);
      if (w < 0) {
        set_abort(bars, a.err);
        break;
      }
      if (w >= n_work) break;
      const Work t = decode_work(a, w, n_mblocks, group_units, kBM);
      if (t.br.nb == 0) continue;
      const bool ok = tma_v256<kAlibi>(&tm_v, smem, bars, t, g, v_issued);
      g += t.br.nb;
      if (!ok) {
        set_abort(bars, a.err);
        break;
      }
    }
    if (v_issued > 0) mbar_wait(&bars->v_full, (v_issued - 1) & 1, kTimeoutNs);
  } else if (warp == kMmaWarp256 && lane == 0) {
    int g = 0, it = 0;
    for (int seq = 0;; ++seq) {
      const int w = sched_take(bars, seq, false);
      if (w < 0) {
        set_abort(bars, a.err);
        break;
      }
      if (w >= n_work) break;
      const Work t = decode_work(a, w, n_mblocks, group_units, kBM);
      if (t.br.nb == 0) continue;
      const bool ok = mma_256<kBF16, kFold>(smem, bars, tmem, t.br.nb, it, g);
      g += t.br.nb;
      ++it;
      if (!ok) {
        set_abort(bars, a.err);
        break;
      }
    }
    tc_commit(&bars->drain);
    mbar_wait(&bars->drain, 0, kTimeoutNs);
  } else if (warp < 4) {
    int g = 0;
    for (int seq = 0;; ++seq) {
      const int w = sched_take(bars, seq, true);
      if (w < 0) {
        set_abort(bars, a.err);
        break;
      }
      if (w >= n_work) break;
      const Work t = decode_work(a, w, n_mblocks, group_units, kBM);
      if (!softmax_256<T, kAlibi, kSoftcap>(a, bars, tmem, warp, t, g)) break;
      g += t.br.nb;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp256) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// -------------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over a [B, S, H, D] tensor given element strides {batch, seq,
// head}, dimensions ordered (D, H, S, B) innermost first, box 64 x 1 x 128 x 1
// (one 128-byte column chunk of 128 rows), 128-byte swizzle, zero fill.
bool make_tile_map(CUtensorMap *m, const void *base, bool bf16, int D, int S, int H, int B,
                   const long long st[3]) {
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return false;
  // A dimension of extent 1 is never stepped along; give it any legal stride.
  auto stride = [](long long elems, int extent) -> cuuint64_t {
    cuuint64_t bytes = (cuuint64_t)elems * 2u;
    if (extent <= 1 && (bytes == 0 || bytes % 16)) bytes = 16;
    return bytes;
  };
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {stride(st[2], H), stride(st[1], S), stride(st[0], B)};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Work-item geometry and grid of one launch: items of `rows` query rows per
// (batch, head) unit, units grouped so a group's K/V (Skv * D * 4 bytes per
// unit) stays within about half of the 126 MB L2; with a work counter one CTA
// per SM (counter zeroed on the stream), else one CTA per item.
struct LaunchShape {
  int n_mblocks, group_units, n_work, grid;
  int *ctr;
};

cudaError_t launch_shape(const AttnArgs &a, int D, int rows, int *work_ctr, cudaStream_t s, LaunchShape *out) {
  const long long n_mblocks = (a.Sq + rows - 1) / rows;
  const long long units = (long long)a.B * a.H;
  // Item indices, and the counter's final values (up to n_work + 2 * grid), stay in int.
  if (n_mblocks * units > 0x7fffffffLL - (1 << 20)) return cudaErrorInvalidValue;
  const long long kv_unit = std::max<long long>(1, (long long)a.Skv * D * 4);
  out->group_units = (int)std::max<long long>(1, std::min<long long>(units, (64ll << 20) / kv_unit));
  out->n_mblocks = (int)n_mblocks;
  out->n_work = (int)(n_mblocks * units);
  const int sms = std::max(1, a.num_sms);
  out->grid = out->n_work;
  out->ctr = nullptr;
  if (work_ctr != nullptr && out->n_work > sms) {
    cudaError_t e = cudaMemsetAsync(work_ctr, 0, sizeof(int), s);
    if (e != cudaSuccess) return e;
    out->grid = sms;
    out->ctr = work_ctr;
  }
  return cudaSuccess;
}

template <typename T, int D, bool kAlibi, bool kSoftcap>
cudaError_t launch_t(const AttnArgs &a, int *work_ctr, cudaStream_t s) {
  using C = Cfg<D>;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap tq, tk, tv;
  if (!make_tile_map(&tq, a.q, bf16, D, a.Sq, a.H, a.B, a.qs) ||
      !make_tile_map(&tk, a.k, bf16, D, a.Skv, a.Hkv, a.B, a.ks) ||
      !make_tile_map(&tv, a.v, bf16, D, a.Skv, a.Hkv, a.B, a.vs))
    return cudaErrorInvalidValue;
  auto kern = fmha_sm100_kernel<T, D, kAlibi, kSoftcap>;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  LaunchShape ls;
  cudaError_t e = launch_shape(a, D, kTiles * kBM, work_ctr, s, &ls);
  if (e != cudaSuccess) return e;
  kern<<<ls.grid, kThreads, C::kSmemBytes, s>>>(tq, tk, tv, a, ls.n_mblocks, ls.group_units, ls.n_work, ls.ctr);
  return cudaGetLastError();
}

template <typename T, bool kAlibi, bool kSoftcap>
cudaError_t launch_t256(const AttnArgs &a, int *work_ctr, cudaStream_t s) {
  using C = Cfg256;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap tq, tk, tv;
  if (!make_tile_map(&tq, a.q, bf16, C::D, a.Sq, a.H, a.B, a.qs) ||
      !make_tile_map(&tk, a.k, bf16, C::D, a.Skv, a.Hkv, a.B, a.ks) ||
      !make_tile_map(&tv, a.v, bf16, C::D, a.Skv, a.Hkv, a.B, a.vs))
    return cudaErrorInvalidValue;
  auto kern = fmha_sm100_d256_kernel<T, kAlibi, kSoftcap>;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return attr_err;
  LaunchShape ls;
  cudaError_t e = launch_shape(a, C::D, kBM, work_ctr, s, &ls);
  if (e != cudaSuccess) return e;
  kern<<<ls.grid, kThreads256, C::kSmemBytes, s>>>(tq, tk, tv, a, ls.n_mblocks, ls.group_units, ls.n_work, ls.ctr);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_d(const AttnArgs &a, int *ctr, cudaStream_t s) {
  const bool alibi = a.alibi != nullptr, cap = a.softcap > 0.f;
  if constexpr (D == 256) {
    if (alibi) return cap ? launch_t256<T, true, true>(a, ctr, s) : launch_t256<T, true, false>(a, ctr, s);
    return cap ? launch_t256<T, false, true>(a, ctr, s) : launch_t256<T, false, false>(a, ctr, s);
  } else {
    if (alibi) return cap ? launch_t<T, D, true, true>(a, ctr, s) : launch_t<T, D, true, false>(a, ctr, s);
    return cap ? launch_t<T, D, false, true>(a, ctr, s) : launch_t<T, D, false, false>(a, ctr, s);
  }
}

}  // namespace

bool sm100_supports(const AttnArgs &a) {
  if (a.dtype != 1 && a.dtype != 2) return false;
  if (a.D != 64 && a.D != 128 && a.D != 256) return false;
  // The softmax takes the row max on raw scores, which needs an increasing
  // score transform (sm_scale > 0); other scales run on the SIMT kernel.
  if (!(a.sm_scale > 0.f)) return false;
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a.q) || !al16(a.k) || !al16(a.v) || !al16(a.o)) return false;
  const long long *st[4] = {a.qs, a.ks, a.vs, a.os};
  for (int t = 0; t < 4; ++t)
    for (int i = 0; i < 3; ++i)
      if (st[t][i] % 8) return false;  // 16-byte strides (TMA, vector stores)
  return true;
}

cudaError_t launch_sm100(const AttnArgs &a, void *ws, size_t ws_bytes, cudaStream_t s) {
  if (!sm100_supports(a)) return cudaErrorNotSupported;
  int *ctr = (ws != nullptr && ws_bytes >= sizeof(int) && (reinterpret_cast<uintptr_t>(ws) & 3u) == 0)
                 ? static_cast<int *>(ws)
                 : nullptr;
  if (a.dtype == 1) {
    if (a.D == 256) return launch_d<__half, 256>(a, ctr, s);
    return a.D == 64 ? launch_d<__half, 64>(a, ctr, s) : launch_d<__half, 128>(a, ctr, s);
  }
  if (a.D == 256) return launch_d<__nv_bfloat16, 256>(a, ctr, s);
  return a.D == 64 ? launch_d<__nv_bfloat16, 64>(a, ctr, s) : launch_d<__nv_bfloat16, 128>(a, ctr, s);
}

}  // namespace llmx_b200
