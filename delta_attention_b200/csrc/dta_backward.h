// Internal launch parameters of the training backward (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace dta {

// Query tiles of the backward are 128 rows = R positions x G heads of one KV
// group (the forward's tile); key tiles are 128 keys.
constexpr int BWD_BN = 128;

enum BwdPass : int { BWD_SPARSE = 0, BWD_DENSE = 1 };

struct BackwardParams {
  CUtensorMap tm_q;     // q (d, s, H, B), box (64, R, G, 1)
  CUtensorMap tm_qsel;  // q of the dense rows, list order (d, n_sel, H, B), box (64, R, G, 1)
  CUtensorMap tm_k;     // k (d, s, Hkv, B), box (64, 128, 1, 1)
  CUtensorMap tm_v;
  CUtensorMap tm_gsp;   // gradient of the sparse rows' output [B, H, s_p, d] as (d, s_p, H, B), box (64, R, G, 1)
  CUtensorMap tm_gdn;   // gradient of the dense rows' output [B, H, n_sel, d], box (64, R, G, 1)
  int B, H, Hkv, G, R, S;
  int s_p, n_anchor, n_sel, gamma, window, sink, qblock;
  float scale_log2;     // scaling * log2(e)
  float scaling;
  const float* lse_sp;  // [B, H, S]: base-2 log-sum-exp of the sparse rows (rows < s_p)
  const float* lse_dn;  // [B, H, n_sel]: of the dense rows
  const float* d_sp;    // [B, H, S]: rowsum(dO * O) of the sparse rows
  const float* d_dn;    // [B, H, n_sel]: of the dense rows
  // query-major launch (dQ): jobs are query tiles of one pass
  int pass;                  // BwdPass of this launch
  int n_qtiles;              // query tiles per (batch, group) of this pass
  __nv_bfloat16* dq;         // [B, H, S, d] bf16 (rows it owns)
  float* dq_dn;              // [B, H, n_anchor, d] fp32: the dense pass's dQ of the anchor rows
  // key-major launch (dK, dV): jobs are chunks of one key tile's query-tile list
  int n_ktiles, chunk_iters, total_chunks;
  const int* chunk_base;     // [n_ktiles + 1]: first chunk of each key tile
  float* dk_acc;             // [B, Hkv, S, d] fp32, accumulated with vector atomics
  float* dv_acc;
  int n_jobs;
  int* counter;              // job counter, zeroed by the host
  int* error;                // kernel error word
  long long wait_cycles;
};

// Query tiles of key tile kt (keys [128 kt, 128 kt + 128)) in the key-major
// launch: sparse query tiles [us0, us1) (rows of R positions below s_p) then
// dense list tiles [ud0, ud1), a superset of the tiles that attend the key tile
// (masked elements contribute nothing).
struct KeyTileList {
  int us0, us1, ud0, ud1;
};

__host__ __device__ inline int bwd_ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// first list index (anchors 0, gamma, ... < s_p, then the tail s_p .. S-1)
// whose position is >= pos
__host__ __device__ inline int bwd_first_list_index(int pos, int gamma, int n_anchor, int s_p) {
  if (pos <= 0) return 0;
  if (n_anchor > 0 && pos <= (n_anchor - 1) * gamma) return bwd_ceil_div(pos, gamma);
  if (pos < s_p) return n_anchor;
  return n_anchor + (pos - s_p);
}

// position of list entry i
__host__ __device__ inline int bwd_list_pos(int i, int gamma, int n_anchor, int s_p) {
  return i < n_anchor ? i * gamma : s_p + (i - n_anchor);
}

// First query position whose window no longer reaches key kv (kv >= sink):
// row t attends kv iff t >= kv and kv > blocklast(t) - window, blocklast(t) =
// (t / qblock) * qblock + qblock - 1, i.e. iff kv <= t < bwd_window_end(kv).
__host__ __device__ inline long long bwd_window_end(long long kv, int window, int qblock) {
  const long long x = kv + window - qblock + 1;
  if (x <= 0) return 0;
  return ((x + qblock - 1) / qblock) * qblock;
}

__host__ __device__ inline KeyTileList bwd_key_tile_list(int kt, int S, int s_p, int n_anchor, int n_sel, int gamma,
                                                         int window, int sink, int qblock, int R) {
  KeyTileList L;
  const long long k0 = (long long)kt * BWD_BN;
  const long long k1 = (k0 + BWD_BN - 1 < S - 1) ? k0 + BWD_BN - 1 : S - 1;
  long long t_end = s_p;
  if (k0 >= sink) {
    const long long e = bwd_window_end(k1, window, qblock);
    if (e < t_end) t_end = e;
  }
  if (t_end > k0) {
    L.us0 = (int)(k0 / R);
    L.us1 = bwd_ceil_div(t_end, R);
  } else {
    L.us0 = L.us1 = 0;
  }
  const int i0 = bwd_first_list_index((int)k0, gamma, n_anchor, s_p);
  if (i0 < n_sel) {
    L.ud0 = i0 / R;
    L.ud1 = bwd_ceil_div(n_sel, R);
  } else {
    L.ud0 = L.ud1 = 0;
  }
  return L;
}

// prep: per anchor block, the delta's gradient and the two passes' output
// gradients, rowsum(dO * O) and the dense rows' q in list order
cudaError_t launch_backward_prep(const __nv_bfloat16* q, long long q_sb, long long q_sh, long long q_ss,
                                 const __nv_bfloat16* out, const __nv_bfloat16* gout, const float* anchor_delta,
                                 __nv_bfloat16* g_sp, __nv_bfloat16* g_dn, __nv_bfloat16* q_sel, float* d_sp,
                                 float* d_dn, int B, int H, int S, int d, int s_p, int n_anchor, int n_sel, int gamma,
                                 float delta_grad_scale, cudaStream_t stream);
cudaError_t launch_backward_plan(int* chunk_base, int n_ktiles, int S, int s_p, int n_anchor, int n_sel, int gamma,
                                 int window, int sink, int qblock, int R, int chunk_iters, cudaStream_t stream);
cudaError_t launch_backward_dq(const BackwardParams& p, int head_dim, int grid, cudaStream_t stream);
// `dependent`: queued as a programmatic dependent launch of the launch before
// it on the stream (its CTAs may start while that grid runs; each waits for it
// before exiting)
cudaError_t launch_backward_dkdv(const BackwardParams& p, int head_dim, int grid, bool dependent, cudaStream_t stream);
// dk = scaling * dk_acc, dv = dv_acc, both to bf16 [B, Hkv, S, d]
cudaError_t launch_backward_finalize(const float* dk_acc, const float* dv_acc, __nv_bfloat16* dk, __nv_bfloat16* dv,
                                     long long n, float scaling, cudaStream_t stream);

}  // namespace dta
