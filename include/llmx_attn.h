/*
 * llmx_attn.h -- C ABI of the B200 (sm_100a) attention forward engine.
 *
 * Plain pointers and sizes only; every entry point returns an llmx_status and
 * allocates nothing.  All device pointers must live on the CUDA device that is
 * current on the calling thread; work is enqueued on the caller's stream.
 *
 * Reference interfaces this ABI replaces (paths inside DucHUNG312/llmx):
 *   llmx_single_mha_attention   include/llmx/cuda/attention/attention_api.h:8-14
 *                               src/cuda/attention/attention_api.cpp:14-72
 *   MHAParams (+ normalize)     include/llmx/cuda/attention/params.h:7-51
 *   single_mha_attention_launcher
 *                               include/llmx/cuda/attention/device/single_mha_kernel.cuh:595-635
 * The reference signature is one causal sequence on stream 0; llmx_attn_fwd
 * adds the batch axis, a non-causal mode, per-sequence lengths (padding),
 * fp32, a caller stream, an optional log-sum-exp output and a caller-owned
 * workspace for split-KV decoding.
 */
#ifndef LLMX_ATTN_H
#define LLMX_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLMX_ATTN_ABI_VERSION 3

#if defined(__GNUC__)
#define LLMX_API __attribute__((visibility("default")))
#else
#define LLMX_API
#endif

typedef enum llmx_status {
  LLMX_OK = 0,
  LLMX_ERR_INVALID_ARGUMENT = 1, /* bad shape, stride, pointer or value      */
  LLMX_ERR_UNSUPPORTED = 2,      /* valid request no kernel here implements  */
  LLMX_ERR_WORKSPACE_TOO_SMALL = 3,
  LLMX_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed     */
  LLMX_ERR_TIMEOUT = 5,          /* a bounded device-side wait expired       */
  LLMX_ERR_NO_DEVICE = 6
} llmx_status;

/* Element types, numbered as llmx::ScalarType (include/llmx/tensor.h:19). */
typedef enum llmx_dtype { LLMX_FP32 = 0, LLMX_FP16 = 1, LLMX_BF16 = 2 } llmx_dtype;

/* Kernel selection.  AUTO picks per request; the others force one family and
 * fail with LLMX_ERR_UNSUPPORTED when it cannot run the request. */
typedef enum llmx_attn_algo {
  LLMX_ALGO_AUTO = 0,
  LLMX_ALGO_SIMT = 1,    /* fp32-accumulating CUDA-core kernel, every shape  */
  LLMX_ALGO_DECODE = 2,  /* split-KV decode, max_q_len == 1, fp16/bf16       */
  LLMX_ALGO_TCGEN05 = 3  /* TMA + tcgen05/TMEM prefill, fp16/bf16, D 64/128/256 */
} llmx_attn_algo;

/*
 * One attention forward over a padded batch.
 *   q, o : [batch, max_q_len,  n_heads,    head_dim]
 *   k, v : [batch, max_kv_len, n_kv_heads, head_dim]
 * given by element strides {batch, seq, head}; the head_dim stride is 1.
 * Sequence b uses its first q_lens[b] query rows and kv_lens[b] keys (NULL
 * means the max extent; device int32 arrays, values are clamped to
 * [0, max]).  Query row i of sequence b attends to key j when
 *   j < kv_len_b,
 *   causal:  j <= i + (kv_len_b - q_len_b)        (bottom-right, mask.h:54-63)
 *   window:  (i + kv_len_b - q_len_b) - j <= sliding_window  (mask.h:60,66)
 * Score = q.k * sm_scale, then tanh(s/cap)*cap if logits_soft_cap > 0
 * (params.h:35-50), then + alibi_slopes[h] * j (mask.h:75-77).
 * Query rows past q_len_b and rows that see no key are written as 0 (their
 * lse as -inf).  GQA: head h reads kv head h / (n_heads / n_kv_heads).
 * With kv_offset / kv_total (below) j is the key's global position.
 */
typedef struct llmx_attn_params {
  int32_t dtype;      /* llmx_dtype of q, k, v and o                    */
  int32_t batch;      /* >= 1                                            */
  int32_t n_heads;    /* >= 1                                            */
  int32_t n_kv_heads; /* >= 1, divides n_heads                           */
  int32_t head_dim;   /* 1..256                                          */
  int32_t max_q_len;  /* >= 1                                            */
  int32_t max_kv_len; /* >= 1                                            */
  int32_t algo;       /* llmx_attn_algo                                  */
  const void *q;
  const void *k;
  const void *v;
  void *o;
  int64_t q_stride[3]; /* elements: batch, seq, head                     */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  const int32_t *q_lens;      /* device [batch] or NULL                  */
  const int32_t *kv_lens;     /* device [batch] or NULL                  */
  const float *alibi_slopes;  /* device [n_heads] fp32 or NULL           */
  float sm_scale;
  int32_t causal;             /* 1 = causal (the reference's only mode)  */
  int32_t sliding_window;     /* < 0 disables                            */
  float logits_soft_cap;      /* <= 0 disables                           */
  float *lse;                 /* NULL or device [batch, n_heads, max_q_len] fp32 */
  void *workspace;            /* device scratch for split-KV partials    */
  size_t workspace_bytes;
  /* Key shards (a sequence's keys split across calls or GPUs): local key j
   * sits at global position kv_offset + j, and the causal / window diagonal
   * of query row i is i + (kv_total - q_len_b) (kv_total <= 0: the local
   * kv_len_b).  ALiBi uses the global position.  Both 0 for unsharded keys. */
  int32_t kv_offset;
  int32_t kv_total;
} llmx_attn_params;

/* Fills *p with defaults: contiguous-stride fields zero, causal = 1,
 * sliding_window = -1, logits_soft_cap = 0, algo = AUTO. */
LLMX_API llmx_status llmx_attn_params_init(llmx_attn_params *p);

/* Sets the four stride triples for contiguous [B, S, H, D] tensors. */
LLMX_API llmx_status llmx_attn_set_contiguous_strides(llmx_attn_params *p);

/* Workspace bytes llmx_attn_fwd wants for *p (0 when none).  A call given
 * less (or NULL) still runs, without splitting the KV axis. */
LLMX_API llmx_status llmx_attn_workspace_size(const llmx_attn_params *p, size_t *bytes);

/* Enqueues the forward on `stream` (a cudaStream_t; NULL = legacy stream).
 * Replaces llmx_single_mha_attention (attention_api.cpp:14-72) for batched,
 * padded and non-causal requests. */
LLMX_API llmx_status llmx_attn_fwd(const llmx_attn_params *p, void *stream);

/* The reference's entry point with plain pointers: one causal sequence,
 * q/o [q_len, n_heads, head_dim], k/v [kv_len, n_kv_heads, head_dim],
 * contiguous.  Same arguments and meaning as
 * llmx::llmx_single_mha_attention (attention_api.h:8-14) plus dtype, the
 * sizes the Tensor carried, and a stream. */
LLMX_API llmx_status llmx_single_mha_attention_c(void *output, const void *q, const void *k, const void *v,
                                        const float *alibi_slopes, int32_t dtype, int32_t q_len,
                                        int32_t kv_len, int32_t n_heads, int32_t n_kv_heads,
                                        int32_t head_dim, float sm_scale, int32_t sliding_window,
                                        float logits_soft_cap, void *stream);

/* Split-KV decode that allocates nothing, for callers that cannot allocate
 * device memory after start-up (a fixed memory budget reserved up front, or a
 * latency-critical loop that must not hit cudaMalloc's implicit device-wide
 * synchronisation) and so cannot pass a workspace.  No counterpart in the
 * reference.  Same request and results as llmx_attn_fwd on the decode path
 * (fp16/bf16, max_q_len == 1, head_dim 64/128/256); the split partials live
 * in one static device array of LLMX_DECODE_NOALLOC_SCRATCH_BYTES per GPU,
 * held by every GPU that loads the library until the process exits.
 *  - Requests needing more scratch than that are refused with
 *    LLMX_ERR_WORKSPACE_TOO_SMALL.  The need is n_splits * batch * n_heads *
 *    (head_dim + 1) * 4 bytes, where a split holds between 64 and 256 keys:
 *    256, halved (down to 64) while batch x kv-head units alone cannot give
 *    the GPU four waves of work, so small batches need up to four times the
 *    256-key figure.  llmx_attn_workspace_size returns the exact need for a
 *    request (the same plan); compare it with the constant below.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current) and keeps it once the
 *    lookup succeeds; a failed lookup is retried on the next call.  Make
 *    that first call before any stream capture.  After cudaDeviceReset the
 *    kept address is stale: do not call this entry point again in that
 *    process.
 *  - All calls on a device share the array: calls that overlap on the GPU
 *    (different streams, or concurrent host threads) race and corrupt each
 *    other's results.  p->workspace is ignored.
 *  - Calls no cudaMalloc, cudaFree or other allocating routine. */
#define LLMX_DECODE_NOALLOC_SCRATCH_BYTES (32u << 20)
LLMX_API llmx_status llmx_attn_decode_noalloc(const llmx_attn_params *p, void *stream);

/* Log-sum-exp merge of attention partials over disjoint key sets (a
 * sequence's keys split across calls or GPUs).  No counterpart in the
 * reference (it has no key splitting); the algebra is its online-softmax
 * rescale (softmax.h:53-110) applied across shards:
 *   m = max_c lse_c,  w_c = exp(lse_c - m),  O = sum_c w_c O_c / sum_c w_c,
 *   lse = m + log(sum_c w_c).
 * Part c covers output rows [row_lo, row_hi) of every (batch, head); for
 * output row s in that range its O element (b, s, h, d) is at
 *   o[b*o_stride[0] + (s - row_lo)*o_stride[1] + h*o_stride[2] + d]
 * and its natural-log lse (-inf: the part saw no key) at
 *   lse[b*lse_stride[0] + h*lse_stride[1] + (s - row_lo)].
 * Rows outside a part's range get no term from it, and a part's O is not
 * read where its lse is -inf, so those rows may hold anything.  Output:
 * out [batch, seq, n_heads, head_dim] with element strides out_stride
 * (batch, seq, head; multiples of 8), in the partials' dtype (fp16/bf16),
 * 0 where no part saw a key; lse_out (NULL or contiguous fp32
 * [batch, n_heads, seq]) = -inf there.  n_parts <= 16; head_dim a
 * multiple of 8; O pointers and strides 16-byte aligned. */
typedef struct llmx_merge_part {
  const void *o;
  const float *lse;
  int64_t o_stride[3];   /* elements: batch, row, head */
  int64_t lse_stride[2]; /* elements: batch, head      */
  int32_t row_lo, row_hi;
} llmx_merge_part;

LLMX_API llmx_status llmx_attn_lse_merge(int32_t n_parts, const llmx_merge_part *parts, int32_t dtype,
                                         int32_t batch, int32_t seq, int32_t n_heads, int32_t head_dim, void *out,
                                         const int64_t *out_stride, float *lse_out, void *stream);

/* Row-scattered partial output: the tensor-core prefill writes query row R
 * (global row row_base + local row) of its partial O and lse into
 * destination p = R / slice_rows, at row R - p * slice_rows of
 *   o[p]   : [batch, slice_rows, n_heads, head_dim] in the input dtype
 *   lse[p] : [batch, n_heads, slice_rows] fp32 (natural log)
 * instead of p->o / p->lse.  The pointers may be another GPU's memory mapped
 * into this process (llmx_ipc_open): a rank of a KV split then delivers each
 * row of its partial straight to the rank that merges that row, while the
 * kernel runs, and every thread fences its writes system-wide before it
 * exits, so a cross-GPU barrier after the launch (an NCCL all-reduce on the
 * same stream) orders them before the owner's merge.  No counterpart in the
 * reference (it has no key splitting).  n_dst <= 8; slice_rows and row_base
 * multiples of 16; every row the launch computes (row_base .. row_base +
 * max_q_len - 1) must fall in a destination; pointers 16-byte aligned. */
#define LLMX_SCATTER_MAX_DST 8
typedef struct llmx_row_scatter {
  int32_t n_dst;
  int32_t slice_rows;
  int32_t row_base;
  int32_t reserved;
  void *o[LLMX_SCATTER_MAX_DST];
  float *lse[LLMX_SCATTER_MAX_DST];
} llmx_row_scatter;

/* llmx_attn_fwd with the output rows scattered as *x describes (p->o and
 * p->lse are ignored).  Runs only on the tensor-core prefill (fp16/bf16,
 * head_dim 64/128); LLMX_ERR_UNSUPPORTED otherwise. */
LLMX_API llmx_status llmx_attn_fwd_scatter(const llmx_attn_params *p, const llmx_row_scatter *x, void *stream);

/* Device buffers shared between the GPUs of one node (one process per GPU)
 * through CUDA IPC, for llmx_attn_fwd_scatter's destinations.  Set-up only,
 * not for the per-call path: llmx_ipc_alloc allocates `bytes` of device
 * memory on the current device (zeroed) and writes its 64-byte IPC handle;
 * another process opens it with llmx_ipc_open (on its own current device, with
 * peer access enabled as needed) and gets a pointer it can store to;
 * llmx_ipc_close unmaps an opened pointer; llmx_ipc_free frees a buffer this
 * process allocated (after every peer has closed it).  Both accept NULL and
 * then do nothing. */
#define LLMX_IPC_HANDLE_BYTES 64
LLMX_API llmx_status llmx_ipc_alloc(size_t bytes, void **ptr, void *handle);
LLMX_API llmx_status llmx_ipc_open(const void *handle, void **ptr);
LLMX_API llmx_status llmx_ipc_close(void *ptr);
LLMX_API llmx_status llmx_ipc_free(void *ptr);

/* Element-type conversion of n contiguous elements between fp32, fp16 and
 * bf16 (round to nearest even), enqueued on `stream`.  Replaces the
 * reference's llmx_copy(ScalarType, ScalarType, ...) (src/tensor.cpp:108-118)
 * and the launch_scalar_convert kernels behind it (src/scalar.cu:33-62),
 * which back the to_fp32 / to_fp16 / to_bf16 ops (include/llmx/ops.h:25-74,
 * 215-229).  fp16 <-> bf16 goes through fp32 as in scalar.cu:6-31.  When the
 * two types match the elements are copied (the reference's same-type
 * converter leaves the output unwritten, include/llmx/scalar.h:13-15).
 * Any pointer alignment is accepted; 16-byte aligned buffers take the
 * vector path. */
LLMX_API llmx_status llmx_convert(const void *src, int32_t src_dtype, void *dst, int32_t dst_dtype, size_t n,
                                  void *stream);

/* Which kernel family llmx_attn_fwd would run for *p (an llmx_attn_algo). */
LLMX_API llmx_status llmx_attn_select_algo(const llmx_attn_params *p, int32_t *algo);

/* Synchronises `device` and reads (and optionally clears) its device-side
 * error word: LLMX_ERR_TIMEOUT if any kernel gave up on a bounded wait. */
LLMX_API llmx_status llmx_attn_device_status(int32_t device, int32_t clear);

LLMX_API const char *llmx_status_string(llmx_status s);
/* Message of the last failing call on this thread ("" if none). */
LLMX_API const char *llmx_attn_last_error(void);
LLMX_API int32_t llmx_attn_abi_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LLMX_ATTN_H */
