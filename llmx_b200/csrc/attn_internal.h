// Internal launch interface shared by the C ABI (attn_api.cu) and the kernel
// translation units.  Host code only sees AttnArgs and the launch_* entry
// points; nothing here is exported from the shared library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "llmx_attn.h"

namespace llmx_b200 {

// Device-side error codes OR-ed into the per-device error word.
enum DeviceError : unsigned int {
  kDevErrTimeout = 1u,   // a bounded mbarrier / flag wait gave up
  kDevErrTmemAlloc = 2u  // tensor-memory allocation did not return in time
};

// A validated, normalised request (all shapes positive, strides in elements).
struct AttnArgs {
  int dtype;  // llmx_dtype
  int B, H, Hkv, D, Sq, Skv, group;
  const void *q, *k, *v;
  void *o;
  long long qs[3], ks[3], vs[3], os[3];  // batch, seq, head
  const int *q_lens, *kv_lens;           // nullable device arrays
  const float *alibi;                    // nullable device [H]
  float sm_scale;
  float softcap;  // <= 0: off
  int causal;
  int window;  // < 0: off
  float *lse;  // nullable [B, H, Sq]
  int kv_offset;  // global position of local key 0
  int kv_total;   // full key length for the causal / window diagonal (0: local)
  unsigned int *err;  // device error word (never null)
  int num_sms;
  // Row-scattered output (llmx_attn_fwd_scatter); xs_n == 0: the usual o / lse.
  int xs_n, xs_slice, xs_row_base;
  void *xs_o[LLMX_SCATTER_MAX_DST];
  float *xs_lse[LLMX_SCATTER_MAX_DST];
};

// Split-KV decode plan: how many splits of how many keys.
struct DecodePlan {
  int chunk;       // keys per split
  int n_splits;    // splits per (batch, kv head)
  int heads_per_cta;
  size_t ws_bytes; // partial O + partial lse
};

DecodePlan plan_decode(const AttnArgs &a, size_t ws_available, bool have_ws);

// Validation shared with entry points outside attn_api.cu: checks *p, that
// the split-KV decode family can run it, and the current device; fills *a
// (error word and SM count included).  Records the message on failure.
llmx_status prepare_decode_request(const llmx_attn_params *p, AttnArgs *a);
llmx_status record_error(llmx_status s, const char *msg);

cudaError_t launch_simt(const AttnArgs &a, cudaStream_t s);
cudaError_t launch_decode(const AttnArgs &a, const DecodePlan &plan, void *ws, cudaStream_t s);
// Returns cudaErrorNotSupported when the request is outside the kernel's
// envelope (dtype, head_dim, alignment); the caller then picks another path.
bool sm100_supports(const AttnArgs &a);
// Workspace the tensor-core prefill uses for its work counter.  Given at
// least that much (4-byte aligned), it runs one CTA per SM over a work queue
// (the counter is zeroed on the stream before the launch); otherwise one CTA
// per work item.
constexpr size_t kSm100WorkspaceBytes = 256;
cudaError_t launch_sm100(const AttnArgs &a, void *ws, size_t ws_bytes, cudaStream_t s);

}  // namespace llmx_b200
