// Delta-attention prefill on sm_100a, double-buffered variant (selected with
// PREFILL_NQ == 1): one persistent, warp-specialised attention kernel used in
// the same two launches per layer as the ping-pong variant ("rows": key-dense
// causal attention for the anchor and tail rows plus key-sparse attention for
// the anchor rows, delta_attention/delta_kernel.py:57-70; "window": key-sparse
// attention for every row below s_p, delta_attention/train/flex_delta.py:59-61,
// with the correction of delta_attention/llama.py:733-757 fused into the
// epilogue).
//
// A job is one 128-row query tile (R rows x G heads of one KV group).  TMEM
// holds two S buffers and two O accumulators, so nothing on the tensor pipe
// waits for the softmax of the same tile:
//   * S(t) for the kernel-wide key-tile sequence t goes to S buffer t % 2; the
//     MMA issuer runs two tiles ahead (S(t + 2) is issued right after PV(t),
//     which consumed the P that aliases S buffer t % 2), so the softmax of
//     tile t + 1 starts as soon as that of tile t ends.
//   * job j accumulates into O buffer j % 2, and a separate epilogue warpgroup
//     normalises, corrects and stores O(j) while the softmax and the MMAs
//     already run job j + 1.
// Three warpgroups (384 threads):
//   warp 0       : producer (job fetch, Q by TMA or cp.async gather, K and V by TMA)
//   warp 1       : TMEM owner; lane 0 issues every tcgen05.mma and commit
//   warps 2, 3   : idle
//   warps 4..7   : softmax, one thread per row (TMEM lane)
//   warps 8..11  : epilogue, one thread per row
// TMEM (512 columns): S0, S1 at columns 0 and 128 (P is written back over the
// first 64 columns of its S buffer as packed bf16 and read by the TS-form MMA),
// O0, O1 at columns 256 and 384.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cmath>
#include <cstddef>

#include "dta_ptx.cuh"
#include "dta_prefill.h"
#include "dta_prefill_jobs.cuh"

#if DTA_PREFILL_NQ == 1
namespace dta {

constexpr int BM = 128;
constexpr int BN = PREFILL_BN;  // keys per tile
static_assert(BN == 128, "S buffers are 128 columns");
constexpr int NUM_THREADS = 384;
constexpr int CTRL_BYTES = 2048;
constexpr int JOB_SLOTS = 2;
#ifndef DTA_POLY_PAIRS
#define DTA_POLY_PAIRS 0
#endif
constexpr int POLY_PAIRS = DTA_POLY_PAIRS;

template <int HD>
struct Geo {
  static constexpr int REGIONS = HD / 64;           // 128-byte swizzle atoms along head_dim
  static constexpr int REGION_BYTES = 128 * 128;    // Q: 128 rows x 128 bytes
  static constexpr int TILE_BYTES = REGIONS * REGION_BYTES;  // one 128 x HD bf16 Q tile
  static constexpr int KV_REGION_BYTES = BN * 128;  // K/V: BN rows x 128 bytes
  static constexpr int KV_TILE_BYTES = REGIONS * KV_REGION_BYTES;
  static constexpr int Q_SLOTS = 2;                 // job j's Q in slot j % 2
  static constexpr int K_STAGES = 2;
  static constexpr int V_STAGES = 2;
  static constexpr int Q_OFF = CTRL_BYTES;
  static constexpr int K_OFF = Q_OFF + Q_SLOTS * TILE_BYTES;
  static constexpr int V_OFF = K_OFF + K_STAGES * KV_TILE_BYTES;
  static constexpr int SMEM_BYTES = V_OFF + V_STAGES * KV_TILE_BYTES + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = 512;
  static constexpr int S_COL = 0;    // S buffer b at b * 128
  static constexpr int O_COL = 256;  // O buffer b at 256 + b * 128
};
static_assert(Geo<128>::SMEM_BYTES <= 232448, "shared memory budget");

struct Ctrl {
  uint64_t job_full[JOB_SLOTS], job_empty[JOB_SLOTS];
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2];        // S buffer b holds a finished S tile
  uint64_t p_full[2][2];     // [S buffer][key half]: that half of P is in TMEM
  uint64_t o_full;           // one phase per PV product (kernel-wide order)
  uint64_t o_done[2];        // O buffer b holds a finished job
  uint64_t o_empty[2];       // the epilogue has read O buffer b
  uint64_t l_ready[2];       // row sums of O buffer b's job are in xl[b]
  uint64_t drain;
  int job[JOB_SLOTS][8];
  uint32_t tmem_base;
  int abort_flag;
  float xl[2][128];          // row sums handed from the softmax to the epilogue
};
static_assert(sizeof(Ctrl) <= CTRL_BYTES, "control block too large");

template <int HD>
__global__ void __launch_bounds__(NUM_THREADS, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  using G = Geo<HD>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(base);
  const uint32_t ctrl_u32 = base_u32;
#define BAR(field) (ctrl_u32 + (uint32_t)offsetof(Ctrl, field))
  const uint32_t q_u32 = base_u32 + G::Q_OFF;
  const uint32_t k_u32 = base_u32 + G::K_OFF;
  const uint32_t v_u32 = base_u32 + G::V_OFF;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &ctrl->abort_flag;
  int* err = p.error;

  if (threadIdx.x == 0) {
    for (int i = 0; i < JOB_SLOTS; ++i) {
      mbar_init(BAR(job_full[0]) + 8 * i, 1);
      mbar_init(BAR(job_empty[0]) + 8 * i, 1 + 4 + 4);  // MMA thread + softmax and epilogue warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(BAR(q_full[0]) + 8 * i, 1);
      mbar_init(BAR(q_empty[0]) + 8 * i, 1);
      mbar_init(BAR(k_full[0]) + 8 * i, 1);
      mbar_init(BAR(k_empty[0]) + 8 * i, 1);
      mbar_init(BAR(v_full[0]) + 8 * i, 1);
      mbar_init(BAR(v_empty[0]) + 8 * i, 1);
      mbar_init(BAR(s_full[0]) + 8 * i, 1);
      mbar_init(BAR(p_full[0][0]) + 8 * (2 * i), 4);
      mbar_init(BAR(p_full[0][0]) + 8 * (2 * i + 1), 4);
      mbar_init(BAR(o_done[0]) + 8 * i, 1);
      mbar_init(BAR(o_empty[0]) + 8 * i, 4);
      mbar_init(BAR(l_ready[0]) + 8 * i, 4);
    }
    mbar_init(BAR(o_full), 1);
    mbar_init(BAR(drain), 1);
    ctrl->abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    if (p.launch == LAUNCH_WINDOW) tma_prefetch_desc(&p.tm_q);
  }
  // Every warp must be converged at a CTA barrier (bar.sync counts whole
  // warps) and at the warp-collective TMEM alloc/dealloc.
  __syncwarp();
  if (warp == 1) {
    tmem_alloc(BAR(tmem_base), G::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  // job slot it % 2, phase (it / 2) & 1: every consumer role reads the same sequence
  auto read_job = [&](int it, Job& J) -> bool {
    const int slot = it & 1;
    if (!mbar_wait_warp(BAR(job_full[0]) + 8 * slot, (it >> 1) & 1, abort_flag, err, KERR_TIMEOUT_SOFTMAX))
      return false;
    const volatile int* src = ctrl->job[slot];
    J.kind = src[0]; J.b = src[1]; J.g = src[2]; J.start = src[3]; J.count = src[4];
    __syncwarp();
    if (lane == 0) mbar_arrive(BAR(job_empty[0]) + 8 * slot);
    return true;
  };

  if (warp == 0) {
    // ======================= producer =======================
    int n = 0;  // K/V tiles issued so far (kernel-wide sequence)
    bool ok = true;
    for (int it = 0; ok; ++it) {
      const int slot = it & 1;
      int j;
      if (p.launch == LAUNCH_WINDOW) {
        j = blockIdx.x + it * gridDim.x;
      } else {
        int jj = 0;
        if (lane == 0) jj = atomicAdd(p.counter, 1);
        j = __shfl_sync(0xffffffffu, jj, 0);
      }
      if (!mbar_wait_warp(BAR(job_empty[0]) + 8 * slot, ((it >> 1) & 1) ^ 1, abort_flag, err,
                          KERR_TIMEOUT_PRODUCER))
        break;
      const Job J = decode_job(p, j);
      if (lane == 0) {
        int* dst = ctrl->job[slot];
        dst[0] = J.kind; dst[1] = J.b; dst[2] = J.g; dst[3] = J.start; dst[4] = J.count;
        mbar_arrive(BAR(job_full[0]) + 8 * slot);
      }
      if (J.kind == JOB_END) break;
      const Plan P = make_plan(p, J);
      // ---- Q of job `it` into slot it % 2, freed by job it-2's last S ----
      {
        const int qs = it & 1;
        const uint32_t qbuf = q_u32 + (uint32_t)qs * G::TILE_BYTES;
        if (!mbar_wait_warp(BAR(q_empty[0]) + 8 * qs, ((it >> 1) & 1) ^ 1, abort_flag, err, KERR_TIMEOUT_PRODUCER))
          break;
        if (J.kind == JOB_WINDOW) {
          if (lane == 0) {
            mbar_arrive_expect_tx(BAR(q_full[0]) + 8 * qs, G::TILE_BYTES);
            for (int r = 0; r < G::REGIONS; ++r)
              tma_load_4d(qbuf + r * G::REGION_BYTES, &p.tm_q, BAR(q_full[0]) + 8 * qs, r * 64, J.start, J.g * p.G,
                          J.b);
          }
        } else {
          // gather R list rows x G heads with cp.async into the 128-byte-
          // swizzled K-major layout the MMA expects
          constexpr int CH = HD / 8;  // 16-byte chunks per row
          const __nv_bfloat16* qb = p.q + (long long)J.b * p.q_sb;
          for (int c = lane; c < BM * CH; c += 32) {
            const int m = c / CH, cc = c - (c / CH) * CH;
            const int hh = m / p.R, rr = m - (m / p.R) * p.R;
            const bool valid = rr < J.count;
            const int row = valid ? list_q_row(p, J.start + rr) : 0;
            const __nv_bfloat16* src =
                qb + (long long)(J.g * p.G + hh) * p.q_sh + (long long)row * p.q_ss + cc * 8;
            const int region = cc >> 3, cw = cc & 7;
            const uint32_t dst = qbuf + region * G::REGION_BYTES + m * 128 + ((cw ^ (m & 7)) << 4);
            cp_async_16(dst, src, valid ? 16u : 0u);
          }
          cp_async_wait_all();
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(BAR(q_full[0]) + 8 * qs);
        }
      }
      // ---- K and V tiles ----
      for (int i = 0; i < P.n_tiles; ++i, ++n) {
        const int st = n & 1;
        const uint32_t ph = (uint32_t)((n >> 1) & 1);
        const int ks = tile_key_start(P, i);
        if (!mbar_wait_warp(BAR(k_empty[0]) + 8 * st, ph ^ 1, abort_flag, err, KERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t kdst = k_u32 + (uint32_t)st * G::KV_TILE_BYTES;
          mbar_arrive_expect_tx(BAR(k_full[0]) + 8 * st, G::KV_TILE_BYTES);
          for (int r = 0; r < G::REGIONS; ++r)
            tma_load_4d(kdst + r * G::KV_REGION_BYTES, &p.tm_k, BAR(k_full[0]) + 8 * st, r * 64, ks, J.g, J.b);
        }
        if (!mbar_wait_warp(BAR(v_empty[0]) + 8 * st, ph ^ 1, abort_flag, err, KERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t vdst = v_u32 + (uint32_t)st * G::KV_TILE_BYTES;
          mbar_arrive_expect_tx(BAR(v_full[0]) + 8 * st, G::KV_TILE_BYTES);
          for (int r = 0; r < G::REGIONS; ++r)
            tma_load_4d(vdst + r * G::KV_REGION_BYTES, &p.tm_v, BAR(v_full[0]) + 8 * st, r * 64, ks, J.g, J.b);
        }
      }
    }
    // On abort, let in-flight TMA loads land before the CTA can exit.
    if (*abort_flag && lane == 0) {
      for (int m = max(0, n - 2); m < n; ++m) {
        const int st = m & 1;
        const uint32_t ph = (uint32_t)((m >> 1) & 1);
        const long long t0 = clock64();
        while (!(mbar_try_wait(BAR(k_full[0]) + 8 * st, ph) && mbar_try_wait(BAR(v_full[0]) + 8 * st, ph))) {
          if (clock64() - t0 > kWaitTimeoutCycles) break;
        }
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, BN, 0);
      constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, HD, 1);
      const uint64_t qdesc0 = smem_desc_sw128(q_u32, 16, 1024);
      const uint64_t kdesc0 = smem_desc_sw128(k_u32, 16, 1024);
      const uint64_t vdesc0 = smem_desc_sw128(v_u32, G::KV_REGION_BYTES, 1024);
      // Two cursors over the kernel-wide key-tile sequence: S runs two tiles
      // ahead of PV.  Tile counts of the jobs between them sit in a ring.
      int ring_T[4] = {0, 0, 0, 0};
      int jobs_read = 0;            // jobs fetched by the S cursor
      int s_job = -1, s_i = 0, s_T = 0, s_t = 0;  // S cursor: job, tile in job, tiles in job, kernel-wide tile
      bool s_end = false;
      int p_job = 0, p_i = 0, p_t = 0;            // PV cursor
      bool aborted = false;
      auto issue_s = [&]() -> bool {
        if (s_end) return true;
        if (s_job < 0 || s_i == s_T) {
          Job J;
          const int it = jobs_read;
          const int slot = it & 1;
          if (!mbar_poll(BAR(job_full[0]) + 8 * slot, (it >> 1) & 1, abort_flag, err, KERR_TIMEOUT_MMA)) return false;
          {
            const volatile int* src = ctrl->job[slot];
            J.kind = src[0]; J.b = src[1]; J.g = src[2]; J.start = src[3]; J.count = src[4];
          }
          mbar_arrive(BAR(job_empty[0]) + 8 * slot);
          if (J.kind == JOB_END) {
            s_end = true;
            return true;
          }
          const Plan P = make_plan(p, J);
          ++jobs_read;
          s_job = it;
          s_i = 0;
          s_T = P.n_tiles;
          ring_T[it & 3] = s_T;
        }
        const int qs = s_job & 1;
        if (s_i == 0) {
          if (!mbar_poll(BAR(q_full[0]) + 8 * qs, (s_job >> 1) & 1, abort_flag, err, KERR_TIMEOUT_MMA)) return false;
        }
        const int st = s_t & 1;
        if (!mbar_poll(BAR(k_full[0]) + 8 * st, (s_t >> 1) & 1, abort_flag, err, KERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t tS = tmem + G::S_COL + (uint32_t)st * BN;  // S buffer t % 2
        // descriptors differ only in the 14-bit start-address field, which
        // never carries out (shared memory < 256 KB), so offsets are plain adds
        const uint64_t qd = qdesc0 + (((uint32_t)qs * G::TILE_BYTES) >> 4);
        const uint64_t kd = kdesc0 + (((uint32_t)st * G::KV_TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qoff = ((kk >> 2) * G::REGION_BYTES + (kk & 3) * 32) >> 4;
          const uint32_t koff = ((kk >> 2) * G::KV_REGION_BYTES + (kk & 3) * 32) >> 4;
          umma_ss(tS, qd + qoff, kd + koff, IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(BAR(s_full[0]) + 8 * st);
        umma_commit(BAR(k_empty[0]) + 8 * st);
        if (s_i == s_T - 1) umma_commit(BAR(q_empty[0]) + 8 * qs);
        ++s_i;
        ++s_t;
        return true;
      };
      // O(job) += P(t) . V(t), in two halves of the key tile
      auto issue_pv = [&]() -> bool {
        const int sb = p_t & 1;
        const uint32_t ph = (uint32_t)((p_t >> 1) & 1);
        const int ob = p_job & 1;
        const uint32_t pbar = BAR(p_full[0][0]) + 8 * (2 * sb);
        if (!mbar_poll(pbar, ph, abort_flag, err, KERR_TIMEOUT_MMA)) return false;
        if (p_i == 0 && p_job >= 2) {
          // the epilogue of job p_job - 2 has read this O buffer
          if (!mbar_poll(BAR(o_empty[0]) + 8 * ob, ((p_job >> 1) - 1) & 1, abort_flag, err, KERR_TIMEOUT_MMA))
            return false;
        }
        if (!mbar_poll(BAR(v_full[0]) + 8 * sb, ph, abort_flag, err, KERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t tP = tmem + G::S_COL + (uint32_t)sb * BN;
        const uint32_t tO = tmem + G::O_COL + (uint32_t)ob * 128;
        const uint64_t vd = vdesc0 + (((uint32_t)sb * G::KV_TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < BN / 32; ++kk)
          umma_ts(tO, tP + kk * 8, vd + ((kk * 2048) >> 4), IDESC_PV, (p_i == 0 && kk == 0) ? 0u : 1u);
        if (!mbar_poll(pbar + 8, ph, abort_flag, err, KERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = BN / 32; kk < BN / 16; ++kk) umma_ts(tO, tP + kk * 8, vd + ((kk * 2048) >> 4), IDESC_PV, 1u);
        umma_commit(BAR(o_full));
        umma_commit(BAR(v_empty[0]) + 8 * sb);
        if (p_i == ring_T[p_job & 3] - 1) {
          umma_commit(BAR(o_done[0]) + 8 * ob);
          ++p_job;
          p_i = 0;
        } else {
          ++p_i;
        }
        ++p_t;
        return true;
      };
      // prologue: S of the first two tiles, then PV(t), S(t + 2), ...
      if (!issue_s() || !issue_s()) aborted = true;
      while (!aborted && p_t < s_t) {
        if (!issue_pv()) {
          aborted = true;
          break;
        }
        if (!issue_s()) aborted = true;
      }
      // drain: every issued tcgen05 op completes before TMEM is released
      umma_commit(BAR(drain));
      const long long t0 = clock64();
      while (!mbar_try_wait(BAR(drain), 0)) {
        if (clock64() - t0 > kWaitTimeoutCycles) {
          atomicCAS(err, 0, KERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ======================= softmax =======================
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;    // row of this thread inside the query tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int rr = r - (r / p.R) * p.R;
    const float sl2 = p.scale_log2;
    int cnt = 0;  // S tiles consumed (kernel-wide sequence)
    for (int it = 0;; ++it) {
      Job J;
      if (!read_job(it, J)) break;
      if (J.kind == JOB_END) break;
      const Plan P = make_plan(p, J);
      const int T = P.tiles_t[0];
      const int ob = it & 1;
      const uint32_t tO = tmem + lane_off + G::O_COL + (uint32_t)ob * 128;
      const bool row_valid = rr < J.count;
      const int qpos = row_valid ? job_row_pos(p, J, rr) : P.qmax_t[0];
      const bool sparse_kind = (J.kind != JOB_DENSE_ROWS);
      const int lo_q = sparse_kind ? block_window_lo(p, qpos) : 0;
      const int sink_q = sparse_kind ? p.sink : 0x7fffffff;
      const int qmin_t = P.qmin_t[0];
      const int lo_max_t = P.lo_max_t[0];

      float m_run = -INFINITY, l_run = 0.f;
      bool aborted = false;
      for (int i = 0; i < T; ++i, ++cnt) {
        const int sb = cnt & 1;
        const uint32_t tS = tmem + lane_off + G::S_COL + (uint32_t)sb * BN;
        if (!mbar_wait_warp(BAR(s_full[0]) + 8 * sb, (cnt >> 1) & 1, abort_flag, err, KERR_TIMEOUT_SOFTMAX)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const int ks = tile_key_start(P, i);
        const int seg_lo = (i < P.n0) ? 0 : P.lo_min;
        const int seg_hi = (i < P.n0) ? P.sink_end : P.qmax + 1;  // exclusive
        const bool full = (ks >= seg_lo) && (ks + BN <= seg_hi) && (ks + BN - 1 <= qmin_t) &&
                          (!sparse_kind || ks + BN <= p.sink || ks >= lo_max_t);
        // load the whole S row (4 x 32 columns) behind a single wait
        float x[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32f(tS + c * 32, x + c * 32);
        tmem_wait_ld();
        if (!full) {
          // column window of this row: valid iff A <= c <= Bq and not X <= c < Y
          const int A = seg_lo - ks;
          const int Bq = min(seg_hi - 1, qpos) - ks;
          const int X = sink_q - ks;
          const int Y = lo_q - ks;
#pragma unroll
          for (int e = 0; e < BN; ++e) {
            const bool v = (e >= A) && (e <= Bq) && !((e >= X) && (e < Y));
            x[e] = v ? x[e] : -INFINITY;
          }
        }
        // row max: 8 independent chains of three-input maxima
        float mk[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float m = fmax3(x[k], x[k + 8], x[k + 16]);
#pragma unroll
          for (int j = 3; j + 1 < BN / 8; j += 2) m = fmax3(m, x[k + 8 * j], x[k + 8 * (j + 1)]);
          mk[k] = fmaxf(m, x[k + BN - 8]);
        }
        float mt = fmax3(fmax3(mk[0], mk[1], mk[2]), fmax3(mk[3], mk[4], mk[5]), fmaxf(mk[6], mk[7]));
        mt *= sl2;  // scaled units (log2 domain); -inf stays -inf
        // keep the running max unless it grows by more than 2^8 (exact: O and
        // l always share the reference max; P stays <= 256)
        const bool need = (i > 0) && (mt > m_run + 8.0f);
        const float m_new = (i == 0 || need) ? mt : m_run;
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        // P = exp2(S * scale - m): scale/shift and row sums on packed fp32
        // pairs; POLY_PAIRS of every 16 pairs take the FMA-pipe exponential
        const uint64_t sc2 = f2_pack(sl2, sl2);
        const uint64_t nm2 = f2_pack(-m_use, -m_use);
        uint64_t ls2[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) ls2[k] = f2_pack(0.f, 0.f);
        auto exp_chunk = [&](int c, uint32_t (&pk)[16]) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float a0, a1, p0, p1;
            f2_unpack(f2_fma(f2_pack(x[c * 32 + 2 * e], x[c * 32 + 2 * e + 1]), sc2, nm2), a0, a1);
            const bool poly = POLY_PAIRS > 0 && (e % 16) * POLY_PAIRS % 16 >= 16 - POLY_PAIRS;
            if (poly) {
              exp2_poly2(a0, a1, p0, p1);
            } else {
              p0 = fast_exp2(a0);
              p1 = fast_exp2(a1);
            }
            ls2[e & 3] = f2_add(ls2[e & 3], f2_pack(p0, p1));
            pk[e] = pack_bf16x2(p0, p1);
          }
        };
        const uint32_t pbar = BAR(p_full[0][0]) + 8 * (2 * sb);
        __syncwarp();  // converge before the warp-collective TMEM stores
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t pk[16];
          exp_chunk(c, pk);
          if (c == BN / 64) {
            // Rescale O when the running max grew by more than 2^8, once
            // PV(t - 1) -- which may still run, S being double-buffered -- is
            // complete; before the first half of P is released, so the whole
            // PV of this tile sees the rescaled O.  The TMEM round trip is
            // warp-collective: lanes that keep their max scale by 1.
            if (i > 0 && __any_sync(0xffffffffu, need)) {
              if (!mbar_wait_warp(BAR(o_full), (cnt - 1) & 1, abort_flag, err, KERR_TIMEOUT_SOFTMAX)) {
                aborted = true;
                break;
              }
              tc_fence_after();
              const float alpha = !need ? 1.f : ((m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new));
#pragma unroll 1
              for (int c2 = 0; c2 < HD / 32; ++c2) {
                float o[32];
                tmem_ld32f(tO + c2 * 32, o);
                tmem_wait_ld();
                uint32_t u[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(o[e] * alpha);
                tmem_st32(tO + c2 * 32, u);
              }
              if (need) l_run *= alpha;
            }
            // the first half of P (keys [0, BN/2)) is in TMEM: release it
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(pbar);
          }
          tmem_st16(tS + c * 16, pk);
        }
        if (aborted) break;
        m_run = m_new;
        {
          float l0, l1;
          f2_unpack(f2_add(f2_add(ls2[0], ls2[1]), f2_add(ls2[2], ls2[3])), l0, l1);
          l_run += l0 + l1;
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pbar + 8);
      }
      if (aborted) break;
      // hand the row sums of this job to the epilogue; xl[ob] is free once the
      // epilogue of job it - 2 has read its O (and, before that, its sums) --
      // a job of one or two key tiles can get here before that epilogue ran
      if (it >= 2 &&
          !mbar_wait_warp(BAR(o_empty[0]) + 8 * ob, ((it >> 1) - 1) & 1, abort_flag, err, KERR_TIMEOUT_SOFTMAX))
        break;
      ctrl->xl[ob][r] = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(l_ready[0]) + 8 * ob);
    }
  } else if (warp >= 8) {
    // ======================= epilogue =======================
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int hh = r / p.R, rr = r - (r / p.R) * p.R;
    for (int it = 0;; ++it) {
      Job J;
      if (!read_job(it, J)) break;
      if (J.kind == JOB_END) break;
      const int ob = it & 1;
      const uint32_t ph = (uint32_t)((it >> 1) & 1);
      const uint32_t tO = tmem + lane_off + G::O_COL + (uint32_t)ob * 128;
      const bool row_valid = rr < J.count;
      const int qpos = row_valid ? job_row_pos(p, J, rr) : 0;
      const int h = J.g * p.G + hh;
      const int gli = J.start + rr;  // list index (row jobs)
      bool store = row_valid;
      int mode_out = 0;  // 0: bf16 to out, 1: fp32 to dense_buf, 2: fp32 to sparse_buf
      long long out_row = 0;
      const __nv_bfloat16* dlt = nullptr;
      if (J.kind == JOB_WINDOW) {
        out_row = qpos;
        if (store && p.mode == 0) {
          int a;
          if (p.anchors) {
            int lo = 0, hi = p.n_anchor - 1;  // last anchor <= qpos (anchors[0] == 0)
            while (lo < hi) {
              const int mid = (lo + hi + 1) >> 1;
              if (p.anchors[mid] <= qpos) lo = mid; else hi = mid - 1;
            }
            a = lo;
          } else {
            a = qpos / p.gamma;
          }
          dlt = p.delta_buf + (((long long)J.b * p.n_anchor + a) * p.H + h) * HD;
        } else if (store && p.mode == 1) {
          bool is_anchor;
          if (p.anchors) {
            int lo = 0, hi = p.n_anchor - 1;
            while (lo < hi) {
              const int mid = (lo + hi + 1) >> 1;
              if (p.anchors[mid] <= qpos) lo = mid; else hi = mid - 1;
            }
            is_anchor = p.anchors[lo] == qpos;
          } else {
            is_anchor = (qpos % p.gamma) == 0;
          }
          store = !is_anchor;
        }
      } else if (J.kind == JOB_DENSE_ROWS) {
        if (gli < p.direct_from) {
          mode_out = 1;
        } else {
          mode_out = 0;
          out_row = !row_valid ? 0 : (p.out_by_list ? gli : list_q_row(p, gli));
        }
      } else {
        mode_out = 2;
      }
      // the owning anchor's delta row (bf16) is fetched before the waits
      uint4 dv[HD / 8];
      if (dlt) {
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) dv[c] = reinterpret_cast<const uint4*>(dlt)[c];
      }
      if (!mbar_wait_warp(BAR(l_ready[0]) + 8 * ob, ph, abort_flag, err, KERR_TIMEOUT_SOFTMAX)) break;
      const float l_tot = ctrl->xl[ob][r];
      if (!mbar_wait_warp(BAR(o_done[0]) + 8 * ob, ph, abort_flag, err, KERR_TIMEOUT_SOFTMAX)) break;
      tc_fence_after();
      const float inv_l = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
      // TMEM reads are warp-collective: every lane loads, stores are predicated
      __nv_bfloat16* dst_bf = (store && mode_out == 0)
                                  ? p.out + (((long long)J.b * p.out_rows + out_row) * p.H + h) * HD
                                  : nullptr;
      float* dst_f = (store && mode_out != 0)
                         ? (mode_out == 1 ? p.dense_buf : p.sparse_buf) +
                               (((long long)J.b * p.n_anchor + gli) * p.H + h) * HD
                         : nullptr;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        __syncwarp();  // stores below are per-lane; converge before the collective load
        tmem_ld32f(tO + c * 32, o);
        tmem_wait_ld();
        if (c == HD / 32 - 1) {
          // O is read: job it + 2 may accumulate into this buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_relaxed(BAR(o_empty[0]) + 8 * ob);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= inv_l;
        if (dst_bf) {
          if (dlt) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              const uint4 w = dv[c * 4 + v4];
              const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                o[v4 * 8 + 2 * k] += __uint_as_float(ww[k] << 16);
                o[v4 * 8 + 2 * k + 1] += __uint_as_float(ww[k] & 0xffff0000u);
              }
            }
          }
#pragma unroll
          for (int e = 0; e < 32; e += 16) {
            uint32_t w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) w[k] = pack_bf16x2(o[e + 2 * k], o[e + 2 * k + 1]);
            st_global_v8(dst_bf + c * 32 + e, w);
          }
        } else if (dst_f) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(dst_f + c * 32 + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
        }
      }
    }
  }
#undef BAR
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Geo<HD>::TMEM_COLS);
  }
}

template <int HD>
static cudaError_t launch_prefill_hd(const PrefillParams& p, int grid, cudaStream_t stream) {
  const int smem = Geo<HD>::SMEM_BYTES;
  cudaError_t e = cudaFuncSetAttribute(prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  prefill_kernel<HD><<<grid, NUM_THREADS, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill(const PrefillParams& p, int head_dim, int grid, cudaStream_t stream) {
  if (head_dim == 128) return launch_prefill_hd<128>(p, grid, stream);
  return launch_prefill_hd<64>(p, grid, stream);
}

}  // namespace dta
#endif  // DTA_PREFILL_NQ == 1
