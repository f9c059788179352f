// llmx's attention op, C++ surface.
//
// llmx_single_mha_attention keeps the reference signature
// (include/llmx/cuda/attention/attention_api.h:8-14): one causal sequence,
// q/o [q_len, n_heads, head_dim], k/v [kv_len, n_kv_heads, head_dim],
// contiguous, optional fp32 ALiBi slopes [n_heads] on the device.  It runs on
// the legacy stream like the reference (attention_api.cpp:55) and throws
// std::runtime_error where the reference's LLMX_CHECK would terminate.
//
// llmx_mha_attention is the extended form the registry and batched callers
// use: [B, S, H, D] tensors, causal flag, per-sequence lengths, a stream and
// an optional lse output.  Both forward to the C ABI in llmx_attn.h.
#pragma once

#include <optional>

#include "llmx/tensor.h"

namespace llmx {

void llmx_single_mha_attention(Tensor &output,                             // [q_len, n_heads, head_dim]
                               const Tensor &q,                            // [q_len, n_heads, head_dim]
                               const Tensor &k,                            // [kv_len, n_kv_heads, head_dim]
                               const Tensor &v,                            // [kv_len, n_kv_heads, head_dim]
                               const std::optional<Tensor> &alibi_slopes,  // [n_heads]
                               float sm_scale, int sliding_window = -1, float logits_soft_cap = 0);

struct MHAOptions {
  bool causal = true;
  int sliding_window = -1;
  float logits_soft_cap = 0.f;
  const int *q_lens = nullptr;   // device int32 [B] or null
  const int *kv_lens = nullptr;  // device int32 [B] or null
  float *lse = nullptr;          // device fp32 [B, H, S_q] or null
  void *stream = nullptr;        // cudaStream_t
};

// q/o [B, S_q, H, D], k/v [B, S_kv, H_kv, D] (3-D tensors are taken as B = 1).
// Split-KV scratch comes from a per-device cache owned by this wrapper.
void llmx_mha_attention(Tensor &output, const Tensor &q, const Tensor &k, const Tensor &v,
                        const std::optional<Tensor> &alibi_slopes, float sm_scale,
                        const MHAOptions &opts = MHAOptions{});

}  // namespace llmx
