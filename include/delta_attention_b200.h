/*
 * delta_attention_b200 — C ABI of the B200 (sm_100a) delta-attention hot path.
 *
 * Plain pointers, sizes and an opaque CUDA stream; no framework types.  Every
 * entry point validates its arguments on the host and returns a dta_status; no
 * exception crosses the boundary.  Kernels never allocate memory: scratch
 * space ("workspace") is provided by the caller, sized by the *_workspace_size
 * query.  All device pointers must be on the current CUDA device.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   dta_prefill  <- LlamaAttention.delta_forward            delta_attention/llama.py:659-757
 *                   (sparse branch hip_attention_interface   delta_attention/llama.py:364-449,
 *                    strided-dense qsa_kernel                 delta_attention/delta_kernel.py:259-329,
 *                    delta broadcast                          delta_attention/llama.py:733-757,
 *                    modes sparse-only / recompute            delta_attention/llama.py:695-696,725-731,
 *                    variable-stride broadcast                delta_attention/stride.py:26-40)
 *   dta_decode   <- LlamaAttention.sdpa_rectangle_forward (s == 1, dense)  delta_attention/llama.py:498-536
 *                   LlamaAttention._decode_sparse_row                      delta_attention/llama.py:538-550
 *                   dense + sparse rows of delta_decode_forward            delta_attention/llama.py:552-634
 *   dta_rows     <- qsa_kernel (attention for a list of query rows, row i
 *                   attending keys [0, limit_i])                 delta_attention/delta_kernel.py:259-329
 *   dta_backward <- autograd of delta_forward_train               delta_attention/train/flex_delta.py:95-196
 */
#ifndef DELTA_ATTENTION_B200_H
#define DELTA_ATTENTION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DTA_ABI_VERSION 3

#if defined(__GNUC__)
#define DTA_API __attribute__((visibility("default")))
#else
#define DTA_API
#endif

typedef enum dta_status {
  DTA_OK = 0,
  DTA_ERR_INVALID_ARG = 1,      /* null pointer, non-positive size, bad enum */
  DTA_ERR_SHAPE = 2,            /* head counts / lengths inconsistent */
  DTA_ERR_STRIDE = 3,           /* stride not a multiple of 16 bytes or head_dim not contiguous */
  DTA_ERR_ALIGNMENT = 4,        /* base pointer not 16-byte aligned */
  DTA_ERR_GAMMA = 5,            /* gamma does not divide s_p, or seq_len < cut_n (the reference's
                                   reshape at delta_attention/llama.py:748-749 would fail) */
  DTA_ERR_HEAD_DIM = 6,         /* head_dim not in the compiled set {64, 128} */
  DTA_ERR_WORKSPACE = 7,        /* workspace missing or smaller than *_workspace_size */
  DTA_ERR_CUDA = 8,             /* a CUDA runtime call failed (see dta_last_cuda_error) */
  DTA_ERR_UNSUPPORTED_DEVICE = 9, /* current device is not sm_100 */
  DTA_ERR_KERNEL_TIMEOUT = 10,  /* a kernel gave up on a bounded wait or met an out-of-range row
                                   (dta_check_workspace / the caller's error_word) */
  DTA_ERR_SCRATCH_LIMIT = 11    /* dta_decode_noalloc: request needs more scratch than its static array */
} dta_status;

typedef enum dta_mode {
  DTA_MODE_DELTA = 0,       /* sparse + (dense - sparse)[anchor]; dense tail rows */
  DTA_MODE_RECOMPUTE = 1,   /* sparse rows, dense rows scattered at anchors and tail */
  DTA_MODE_SPARSE_ONLY = 2  /* sparse rows everywhere */
} dta_mode;

/* Delta-attention prefill of one layer.
 * q: [batch, n_heads, seq_len, head_dim] bf16 (any strides, head_dim contiguous).
 * k, v: [batch, n_kv_heads, seq_len, head_dim] bf16 (same rule).
 * out: [batch, seq_len, n_heads, head_dim] bf16, contiguous (the plug-in's
 *      return layout, delta_attention/llama.py:757).
 * Sparse keys of query row t: kv <= t and (kv < sink or kv > blocklast(t) - window),
 *   blocklast(t) = (t / q_block) * q_block + q_block - 1  (hip-attn block-anchored window).
 * Anchors: uniform stride gamma (cut_n = seq_len % gamma + max(128, gamma),
 *   s_p = seq_len - cut_n, anchors 0, gamma, ... < s_p, dense tail [s_p, seq_len)),
 *   or an explicit sorted device array (anchors[0] == 0, all < s_p) for variable stride. */
typedef struct dta_prefill_args {
  int32_t abi_version; /* DTA_ABI_VERSION */
  int32_t batch, n_heads, n_kv_heads, seq_len, head_dim;
  const void* q;
  int64_t q_stride_b, q_stride_h, q_stride_s; /* in elements */
  const void* k;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  const void* v;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  void* out;
  float scaling;     /* softmax scale, normally head_dim^-0.5 */
  int32_t gamma;     /* Config.delta_lambda: anchor stride */
  int32_t window;    /* Config.sliding_window */
  int32_t sink;      /* attention-sink tokens (reference hard-codes 1024) */
  int32_t q_block;   /* query block of the block-anchored window (reference: 64) */
  int32_t mode;      /* dta_mode */
  const int32_t* anchors; /* optional device array; NULL = uniform stride gamma */
  int32_t n_anchors;      /* length of anchors (when anchors != NULL) */
  int32_t s_p;            /* first dense-tail row (when anchors != NULL) */
  float* anchor_delta;    /* optional out [batch, n_anchor, n_heads, head_dim] fp32:
                             dense - sparse at every anchor (drift telemetry) */
  int32_t phases;         /* 0 = whole prefill; otherwise a mask of DTA_PHASE_* */
  void* workspace;
  size_t workspace_bytes;
  int32_t* error_word;    /* optional device int32: kernels record a timeout or bad-row code
                             here (atomically, first code wins) instead of in the workspace
                             header; never cleared by the library, so it stays set across
                             calls until the caller reads and clears it */
  int64_t wait_cycles;    /* budget of each bounded wait inside the kernels, in SM clock
                             cycles; 0 = the default (~2 s) */
  int32_t flags;          /* mask of DTA_FLAG_* (0 for normal use) */
  int32_t split_tiles;    /* key tiles (128 keys) per split-K chunk of the dense rows; 0 = chosen
                             from the device's SM count and the total work.  A dense row tile
                             longer than this runs as several chunks whose partial results the
                             last-finishing chunk merges (log-sum-exp); see dta_prefill_workspace_size */
  const void* anchor_delta_in; /* optional device bf16 [batch, n_anchors, n_heads, head_dim] with explicit
                             anchors, delta mode: dense - sparse of every anchor row, computed earlier
                             (the adaptive stride planner has it); the ROWS phase then computes only
                             the dense tail rows and WINDOW applies these rows */
  float* lse_sparse;      /* optional out [batch, n_heads, seq_len] fp32: base-2 log-sum-exp of the scaled
                             scores (log2 of the softmax denominator, scores times scaling * log2(e)) of
                             each windowed row's sparse attention, rows [0, s_p) (every row in sparse-only
                             mode; other rows untouched).  Kept by the training forward for dta_backward */
  float* lse_dense;       /* optional out [batch, n_heads, n_sel] fp32: the same for each dense row of the
                             ROWS phase, list order (anchors, then the tail rows s_p .. seq_len-1) */
} dta_prefill_args;

/* Test hook: the producer warp of every CTA first waits on a barrier that
 * nothing ever completes, so that wait runs out after wait_cycles, the CTA
 * abandons its work and the launch records a kernel timeout code.  Lets a
 * test check the timeout path without any faulting or hanging input.
 * Outputs of such a call are not written. */
#define DTA_FLAG_TEST_STALL 1

/* Phases of dta_prefill.  ROWS: dense rows (anchors + tail) and sparse anchor
 * rows, written to the workspace (and anchor_delta when given).  WINDOW: the
 * windowed rows with the fused delta epilogue; it reads what a ROWS call with
 * identical arguments left in the same workspace.  With uniform anchors, 4 or
 * 8 query heads per KV head and gamma a power of two >= 8, WINDOW forms each
 * anchor's sparse row and dense - sparse itself (in the tile that holds the
 * anchor row), so ROWS computes dense rows only and anchor_delta is written by
 * WINDOW. */
#define DTA_PHASE_ROWS 1
#define DTA_PHASE_WINDOW 2

/* Bytes of device workspace dta_prefill needs for these arguments. */
DTA_API size_t dta_prefill_workspace_size(const dta_prefill_args* args);
/* Enqueue the prefill on `stream` (a cudaStream_t; NULL = legacy default). */
DTA_API int dta_prefill(const dta_prefill_args* args, void* stream);

/* Attention for an explicit list of query rows (the qsa_kernel contract):
 * row i takes query q[b, :, q_rows[i]] and attends keys [0, kv_limit[i]];
 * kv_limit must be non-decreasing.  out: [batch, n_rows, n_heads, head_dim]
 * bf16 contiguous.  Used for the sdpa_rectangle (s > 1) continuation rows. */
typedef struct dta_rows_args {
  int32_t abi_version;
  int32_t batch, n_heads, n_kv_heads, seq_len, head_dim, n_rows;
  const void* q;
  int64_t q_stride_b, q_stride_h, q_stride_s;
  const void* k;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  int32_t kv_len;
  const void* v;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  const int32_t* q_rows;   /* device [n_rows] */
  const int32_t* kv_limit; /* device [n_rows], non-decreasing */
  void* out;
  float scaling;
  void* workspace;
  size_t workspace_bytes;
  int32_t* error_word;    /* as in dta_prefill_args */
  int64_t wait_cycles;    /* as in dta_prefill_args */
  int32_t flags;          /* as in dta_prefill_args */
  int32_t split_tiles;    /* as in dta_prefill_args */
} dta_rows_args;
DTA_API size_t dta_rows_workspace_size(const dta_rows_args* args);
DTA_API int dta_rows(const dta_rows_args* args, void* stream);

/* One decode row per (batch, head) over a KV cache of n_keys keys.
 * q: [batch, n_heads, 1, head_dim]; k, v: [batch, n_kv_heads, n_keys(+), head_dim].
 * dense_out / sparse_out: [batch, 1, n_heads, head_dim] bf16 (either may be NULL).
 * Sparse keys: the first `sink` plus the last `window`, or all keys when
 * n_keys <= sink + window.  Both outputs come from ONE pass over the cache. */
typedef struct dta_decode_args {
  int32_t abi_version;
  int32_t batch, n_heads, n_kv_heads, n_keys, head_dim;
  const void* q;
  int64_t q_stride_b, q_stride_h;
  const void* k;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  const void* v;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  float scaling;
  int32_t window, sink;
  void* dense_out;
  void* sparse_out;
  void* workspace;
  size_t workspace_bytes;
  const int32_t* n_keys_dev; /* optional device int32: the live key count, read by the kernels (clamped to
                                [1, n_keys]); n_keys is then the cache capacity the launch is sized for.
                                Lets a CUDA graph replay the same call while the cache grows. */
} dta_decode_args;
DTA_API size_t dta_decode_workspace_size(const dta_decode_args* args);
DTA_API int dta_decode(const dta_decode_args* args, void* stream);

/* dta_decode for callers that cannot allocate device memory.  No counterpart in
 * the reference (it is an addition of this library).
 *
 * Some callers cannot call cudaMalloc where they decode: a serving engine that
 * has handed (nearly) all HBM to its own KV-cache and weight arenas, so a new
 * allocation would fail or bypass the engine's accounting; a program in another
 * language that binds only this C ABI and owns no device allocator; a
 * latency-critical loop in which cudaMalloc/cudaFree would synchronize the device.
 * This entry point ignores args->workspace/workspace_bytes and keeps the split-K
 * partials in a static device array of DTA_DECODE_NOALLOC_SCRATCH_BYTES, which
 * every GPU that loads this library holds until the process exits.
 * - The first call on each device looks up that array's device address (with
 *   that device current) and caches it; make that first call before any stream
 *   capture begins.
 * - A request whose dta_decode_workspace_size exceeds the array is rejected with
 *   DTA_ERR_SCRATCH_LIMIT before anything is launched.
 * - It allocates nothing.  All calls on a device share the one array, which keeps
 *   the last call's contents; nothing in it needs to start at zero (every entry a
 *   call reads was written earlier by the same call).  Calls whose kernels may
 *   overlap on the GPU (different streams, or different host threads) race on the
 *   array: order them on one stream. */
#define DTA_DECODE_NOALLOC_SCRATCH_BYTES (32u << 20)
DTA_API int dta_decode_noalloc(const dta_decode_args* args, void* stream);

/* Training backward of one delta-attention layer with uniform anchors: the
 * gradients of delta_forward_train (delta_attention/train/flex_delta.py:95-196,
 * including its detach_delta / delta_grad_scale arms) with respect to q, k, v.
 * Inputs are the forward's own q, k, v, its output and what a dta_prefill call
 * with anchor_delta, lse_sparse and lse_dense set returned (same gamma, window,
 * sink, q_block and scaling).
 * grad_out: [batch, seq_len, n_heads, head_dim] bf16 contiguous (the output's layout).
 * grad_q: [batch, n_heads, seq_len, head_dim]; grad_k, grad_v: [batch, n_kv_heads,
 * seq_len, head_dim]; all bf16 contiguous.  n_heads / n_kv_heads must be 1, 2, 4 or 8.
 * The workspace (dta_backward_workspace_size) holds the passes' output gradients,
 * row sums and fp32 dK / dV accumulators; dta_check_workspace reads its error word. */
typedef struct dta_backward_args {
  int32_t abi_version;
  int32_t batch, n_heads, n_kv_heads, seq_len, head_dim;
  const void* q;
  int64_t q_stride_b, q_stride_h, q_stride_s;
  const void* k;
  int64_t k_stride_b, k_stride_h, k_stride_s;
  const void* v;
  int64_t v_stride_b, v_stride_h, v_stride_s;
  const void* out;          /* the forward's output */
  const void* grad_out;
  const float* anchor_delta; /* the forward's fp32 dense - sparse per anchor [batch, n_anchor, n_heads, head_dim] */
  const float* lse_sparse;  /* the forward's lse_sparse [batch, n_heads, seq_len] */
  const float* lse_dense;   /* the forward's lse_dense [batch, n_heads, n_sel] */
  void* grad_q;
  void* grad_k;
  void* grad_v;
  float scaling;
  int32_t gamma, window, sink, q_block;
  float delta_grad_scale;   /* factor on the gradient through the broadcast delta (the reference's
                               delta_grad_scale); 0 = the detach_delta arm */
  void* workspace;
  size_t workspace_bytes;
  int32_t* error_word;      /* as in dta_prefill_args */
  int64_t wait_cycles;      /* as in dta_prefill_args */
} dta_backward_args;
DTA_API size_t dta_backward_workspace_size(const dta_backward_args* args);
DTA_API int dta_backward(const dta_backward_args* args, void* stream);

/* Host-side helpers. */
DTA_API int dta_abi_version(void);
DTA_API const char* dta_status_string(int status);
/* Last CUDA runtime error code seen by this thread (0 if none); for a failed TMA
 * tensor-map encode, the driver's CUresult. */
DTA_API int dta_last_cuda_error(void);
/* Synchronously read the kernel error word of a workspace used on `stream`;
 * returns DTA_OK or DTA_ERR_KERNEL_TIMEOUT (kernel code in *kernel_code). */
DTA_API int dta_check_workspace(const void* workspace, void* stream, int* kernel_code);

#ifdef __cplusplus
}
#endif

#endif /* DELTA_ATTENTION_B200_H */
