// Internal launch parameters of the prefill attention kernel (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace dta {

enum Launch : int { LAUNCH_ROWS = 0, LAUNCH_WINDOW = 1 };
// How the windowed launch obtains each anchor's delta (PrefillParams fields
// fuse_delta / delta_pair): from the delta kernel, handed from tile A to tile B
// through shared memory, or formed by the warp holding the anchor row.
enum FuseMode : int { FUSE_NONE = 0, FUSE_PAIR = 1, FUSE_GENERAL = 2 };

// Query tiles (of 128 rows = R rows x G heads) per kernel job: the two tiles
// of a job ping-pong on the tensor core (dta_prefill.cu).
constexpr int PREFILL_NQ = 2;
// Keys per K/V tile (the TMA box height of the K and V tensor maps).
constexpr int PREFILL_BN = 128;

struct PrefillParams {
  CUtensorMap tm_q;  // (d, s, H, B), box (64, R, G, 1): window launch only
  CUtensorMap tm_k;  // (d, s_kv, Hkv, B), box (64, 128, 1, 1)
  CUtensorMap tm_v;
  CUtensorMap tm_out;  // out (d, s, H, B) with box (64, R, G, 1): window launch, when tma_out
  const __nv_bfloat16* q;
  long long q_sb, q_sh, q_ss;  // element strides for the cp.async row gather
  int B, H, Hkv, G, R;
  float scale_log2;             // scaling * log2(e)
  int window, sink, qblock;
  int gamma, s_p, n_anchor, n_sel;
  // n / qblock and n / gamma as multiply-shift (fast_div): integer division
  // would go through the reciprocal unit that the exponentials keep busy
  unsigned long long qblock_mul, gamma_mul;
  int qblock_sh, gamma_sh;
  const int* anchors;           // optional explicit anchor rows (sorted)
  const int* q_rows;            // optional explicit row list (rows launch)
  const int* kv_limit;          // optional explicit key limits (rows launch)
  int mode;                     // 0 delta, 1 recompute, 2 sparse-only
  int launch;                   // Launch
  int row_end;                  // window launch: rows [0, row_end) are produced
  int direct_from;              // rows launch: list index from which dense rows go to `out`
  int out_by_list;              // rows launch: out row = list index (dta_rows) instead of q row
  int out_rows;                 // rows of `out` per batch
  int n_dense_tiles, n_sparse_tiles, n_window_tiles;
  int n_jobs;
  int* counter;                 // job counter (rows launch), zeroed by the host
  int* error;                   // kernel error word, zeroed by the host
  float* dense_buf;             // [B, n_anchor, H, d] fp32
  float* sparse_buf;            // [B, n_anchor, H, d] fp32
  __nv_bfloat16* delta_buf;     // [B, n_anchor, H, d] bf16: dense - sparse (window launch)
  // window launch: form delta = dense - sparse inside the kernel from each
  // anchor row's own sparse output (uniform anchors, 4 or 8 heads per KV
  // group, gamma a power of two >= 8); the rows launch then computes no sparse
  // anchor rows and no delta kernel runs.  delta_cross: anchors are more than
  // R rows apart, so the first job of each anchor period forms them (tile A)
  // for the other tiles of the period; win_group: jobs per anchor period when
  // it spans several (processed consecutively by one CTA), else 1.
  int fuse_delta, delta_cross, win_group;
  // pair delta (gamma = 2R = 64 with 4 heads per group): tile A hands the four
  // heads' delta rows to tile B through shared memory instead of the delta buffer
  int delta_pair;
  float* anchor_delta_f32;      // optional fp32 dense - sparse per anchor (telemetry)
  __nv_bfloat16* out;           // [B, out_rows, H, d]
  int tma_out;                  // window launch: full tiles leave through tm_out (TMA stores)
  // Split-K of the rows launch's dense jobs.  A dense job (one row tile of the
  // list) whose key range spans T > split_c tiles runs as c = ceil(T / split_c)
  // jobs ("chunks") over key tiles [k split_c, (k+1) split_c); each chunk stores its
  // rows' O / l and log2-sum-exp as partials, and the chunk that finishes last
  // (per query tile and warp, counted in part_cnt) merges them and stores the
  // rows.  split_c == 0: no split (one chunk per row tile).  The job index
  // space reserves split_cmax chunks per row tile; chunks past a short tile's
  // c are skipped by the producer.
  int split_c, split_cmax;
  float* part_o;                // [B*Hkv][n_dense_tiles][split_cmax][NQ][d/4][128] float4
  float* part_lse;              // [B*Hkv][n_dense_tiles][split_cmax][NQ][128]
  int* part_cnt;                // [B*Hkv][n_dense_tiles][NQ][4 warps] chunks finished, zeroed by the host
  long long wait_cycles;        // budget of each bounded wait (clock64 cycles, > 0)
  int test_stall;               // test hook: the producer first waits on a barrier nothing completes
  int seq_q, kv_len;            // rows of q and of k/v: bounds for explicit row lists
  // optional base-2 log-sum-exp of every produced row (training forward):
  // windowed rows into lse_sparse[(b * H + h) * seq_q + row], dense rows of the
  // rows launch into lse_dense[(b * H + h) * n_sel + list index]
  float* lse_sparse;
  float* lse_dense;
};

// Multiplier and shift with n / d == (n * mul) >> sh for every 0 <= n < 2^31
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994: mul = ceil(2^(31 + l) / d), l = ceil(log2 d)).
inline void fast_div_params(int d, unsigned long long* mul, int* sh) {
  int l = 0;
  while ((1LL << l) < (long long)d) ++l;
  const unsigned long long num = 1ULL << (31 + l);
  *mul = (num + (unsigned long long)d - 1) / (unsigned long long)d;
  *sh = 31 + l;
}
__device__ __forceinline__ int fast_div(int n, unsigned long long mul, int sh) {
  return (int)(((unsigned long long)(unsigned)n * mul) >> sh);
}

// `dependent`: the windowed launch may start while the rows launch queued just
// before it on the stream is still running (programmatic dependent launch); it
// waits for that grid before reading its output.
cudaError_t launch_prefill(const PrefillParams& p, int head_dim, int grid, bool dependent, cudaStream_t stream);
// delta = dense - sparse per anchor: bf16 into delta_bf16 (for the windowed
// launch) and, when delta_f32 is not null, fp32 into delta_f32 (telemetry).
cudaError_t launch_anchor_delta(const float* dense, const float* sparse, __nv_bfloat16* delta_bf16, float* delta_f32,
                                long long n, cudaStream_t stream);

}  // namespace dta
