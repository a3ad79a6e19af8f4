// Jobs and key-tile plans of the prefill kernel (device code identical in
// every role of the kernel).
#pragma once

#include "dta_prefill.h"
#include "dta_ptx.cuh"

namespace dta {

enum JobKind : int { JOB_END = -1, JOB_WINDOW = 0, JOB_DENSE_ROWS = 1, JOB_SPARSE_ROWS = 2 };

struct Job {
  int kind, b, g, start, count;
  int chunk;  // dense row jobs: key-range chunk of the row tile
};

// ---------------------------------------------------------------------------
// row lists, jobs and key-tile plans (identical in every role)
// ---------------------------------------------------------------------------
// A list entry outside the tensors is recorded in the error word and clamped,
// so a bad caller array costs a wrong (flagged) output, never a stray access.
__device__ __forceinline__ int clamp_row(const PrefillParams& p, int row, int n) {
  if (row < 0 || row >= n) {
    atomicCAS(p.error, 0, KERR_BAD_ROW);
    row = min(max(row, 0), n - 1);
  }
  return row;
}
__device__ __forceinline__ int list_q_row(const PrefillParams& p, int i) {
  if (p.q_rows) return p.q_rows[i];
  if (i < p.n_anchor) return p.anchors ? p.anchors[i] : i * p.gamma;
  return p.s_p + (i - p.n_anchor);
}
__device__ __forceinline__ int list_kv_limit(const PrefillParams& p, int i) {
  return clamp_row(p, p.kv_limit ? p.kv_limit[i] : list_q_row(p, i), p.kv_len);
}

// Job index -> job.  Window launch: (batch x group)-major R*NQ-row tiles of
// rows [0, row_end).  Rows launch: dense row tiles longest first (each with
// split_cmax chunk slots), then sparse anchor tiles; without split-K the
// batch x group index varies fastest, with it the order is group-major.
static __device__ Job decode_job(const PrefillParams& p, int j) {
  Job J;
  const int JR = PREFILL_NQ * p.R;  // rows per job
  J.chunk = 0;
  if (j >= p.n_jobs) {
    J.kind = JOB_END;
    J.b = J.g = J.start = J.count = 0;
    return J;
  }
  if (p.launch == LAUNCH_WINDOW) {
    const int nt = p.n_window_tiles;
    const int bg = j / nt, t = j - bg * nt;
    J.kind = JOB_WINDOW;
    J.b = bg / p.Hkv;
    J.g = bg - J.b * p.Hkv;
    J.start = t * JR;
    J.count = min(JR, p.row_end - J.start);
    return J;
  }
  const int BG = p.B * p.Hkv;
  const int cmax = p.split_cmax > 0 ? p.split_cmax : 1;
  int u, bg;
  if (cmax > 1) {
    // split: group-major (all CTAs sweep one group's K/V together, so each
    // key chunk is read from DRAM about once); the chunks are short enough
    // that the longest-first order inside each group keeps the SMs balanced
    const int per_bg = p.n_dense_tiles * cmax + p.n_sparse_tiles;
    bg = j / per_bg;
    u = j - bg * per_bg;
  } else {
    // whole row tiles: longest first across groups (the longest tiles bound
    // the launch and must start first)
    u = j / BG;
    bg = j - u * BG;
  }
  J.b = bg / p.Hkv;
  J.g = bg - J.b * p.Hkv;
  if (u < p.n_dense_tiles * cmax) {
    const int rank = u / cmax;
    const int tile = p.n_dense_tiles - 1 - rank;  // longest (latest rows) first
    J.kind = JOB_DENSE_ROWS;
    J.chunk = u - rank * cmax;
    J.start = tile * JR;
    J.count = min(JR, p.n_sel - J.start);
  } else {
    const int tile = u - p.n_dense_tiles * cmax;
    J.kind = JOB_SPARSE_ROWS;
    J.start = tile * JR;
    J.count = min(JR, p.n_anchor - J.start);
  }
  return J;
}

// position (key limit) of job-local row r (< J.count)
__device__ __forceinline__ int job_row_pos(const PrefillParams& p, const Job& J, int r) {
  if (J.kind == JOB_WINDOW) return J.start + r;
  return list_kv_limit(p, J.start + r);
}

// index of the anchor that owns row t: the last anchor row <= t (anchor 0 is row 0)
__device__ __forceinline__ int anchor_of(const PrefillParams& p, int t) {
  if (!p.anchors) return fast_div(t, p.gamma_mul, p.gamma_sh);
  int lo = 0, hi = p.n_anchor - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.anchors[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}
__device__ __forceinline__ bool is_anchor_row(const PrefillParams& p, int t) {
  if (!p.anchors) return t == fast_div(t, p.gamma_mul, p.gamma_sh) * p.gamma;
  return p.anchors[anchor_of(p, t)] == t;
}

__device__ __forceinline__ int block_window_lo(const PrefillParams& p, int t) {
  const int bl = fast_div(t, p.qblock_mul, p.qblock_sh) * p.qblock + p.qblock - 1;
  return max(0, bl - p.window + 1);
}

// Key tiles of a job: sink segment [0, sink_end) then window segment
// [lo_min, qmax]; dense jobs have the one segment [lo_min, ...) of their
// chunk (lo_min = 0 when unsplit).  Query tile q takes the prefix of tiles
// whose first key is <= the tile's last row.
struct Plan {
  int n0, n_tiles, sink_end, lo_min, qmax;
  int chunk, n_chunks;  // dense jobs: this chunk and the row tile's chunk count
  int qmin_t[PREFILL_NQ], qmax_t[PREFILL_NQ], lo_max_t[PREFILL_NQ], tiles_t[PREFILL_NQ];
  int act_t[PREFILL_NQ];  // dense jobs: chunks in which query tile q has keys (a prefix)
};

__device__ __forceinline__ int tile_key_start(const Plan& P, int i) {
  return i < P.n0 ? i * PREFILL_BN : P.lo_min + (i - P.n0) * PREFILL_BN;
}

static __device__ Plan make_plan(const PrefillParams& p, const Job& J) {
  Plan P;
  const bool dense = (J.kind == JOB_DENSE_ROWS);
  int first = -1;
  P.qmax = 0;
  P.chunk = J.chunk;
  P.n_chunks = 1;
#pragma unroll
  for (int q = 0; q < PREFILL_NQ; ++q) {
    P.act_t[q] = 1;
    const int r0 = q * p.R;
    const int r1 = min(J.count, (q + 1) * p.R) - 1;
    if (r1 < r0) {
      P.qmin_t[q] = 0;
      P.qmax_t[q] = -1;
      P.lo_max_t[q] = 0;
      continue;
    }
    P.qmin_t[q] = job_row_pos(p, J, r0);
    P.qmax_t[q] = job_row_pos(p, J, r1);
    P.lo_max_t[q] = dense ? 0 : block_window_lo(p, P.qmax_t[q]);
    if (first < 0) first = P.qmin_t[q];
    P.qmax = max(P.qmax, P.qmax_t[q]);
  }
  if (dense) {
    // key tiles [kb, ke) of this chunk out of the row tile's T.  Chunk
    // boundaries are multiples of split_c for every row tile, so chunk k of
    // all row tiles (running at about the same time, longest-first order)
    // read the same key range of their group and share it in L2.
    const int T = P.qmax / PREFILL_BN + 1;
    int c = 1, kb = 0, ke = T;
    if (p.split_c > 0 && T > p.split_c) {
      c = min((T + p.split_c - 1) / p.split_c, p.split_cmax);
      kb = J.chunk * p.split_c;
      ke = (J.chunk == c - 1) ? T : kb + p.split_c;
    }
    P.n_chunks = c;
    P.n0 = 0;
    P.sink_end = 0;
    if (J.chunk >= c) {
      // a chunk slot past this (short) row tile's chunks: an empty job
      P.lo_min = 0;
      P.n_tiles = 0;
#pragma unroll
      for (int q = 0; q < PREFILL_NQ; ++q) P.tiles_t[q] = 0;
      return P;
    }
    P.lo_min = kb * PREFILL_BN;
    P.n_tiles = ke - kb;
#pragma unroll
    for (int q = 0; q < PREFILL_NQ; ++q) {
      const int m = P.qmax_t[q];
      if (m < 0) {
        P.tiles_t[q] = 0;
        continue;
      }
      const int Tq = m / PREFILL_BN + 1;
      P.tiles_t[q] = min(max(Tq - kb, 0), ke - kb);
      // chunk k' has keys for tile q iff it starts below Tq: k' split_c < Tq
      P.act_t[q] = (c == 1) ? 1 : min(c, (Tq + p.split_c - 1) / p.split_c);
    }
    return P;
  }
  P.lo_min = block_window_lo(p, first);
  P.sink_end = min(p.sink, P.lo_min);
  P.n0 = (P.sink_end + PREFILL_BN - 1) / PREFILL_BN;
  P.n_tiles = P.n0 + (P.qmax - P.lo_min) / PREFILL_BN + 1;
#pragma unroll
  for (int q = 0; q < PREFILL_NQ; ++q) {
    const int m = P.qmax_t[q];
    if (m < 0) P.tiles_t[q] = 0;
    else if (m >= P.lo_min) P.tiles_t[q] = P.n0 + (m - P.lo_min) / PREFILL_BN + 1;
    else P.tiles_t[q] = min(P.n0, m / PREFILL_BN + 1);
  }
  return P;
}

}  // namespace dta
