// Delta-attention prefill on sm_100a: one persistent, warp-specialised
// attention kernel used in two launches per layer.
//
//   launch "rows"   : key-dense causal attention for an explicit list of query
//                     rows (anchors + dense tail; the qsa_kernel contract of
//                     delta_attention/delta_kernel.py:57-70) and, unless the
//                     window launch forms the delta itself (fuse_delta), key-
//                     sparse attention for the anchor rows.  Jobs are ordered
//                     longest-first and fetched from an atomic counter, so the
//                     triangular work of the anchor rows balances over the SMs
//                     without split-K.
//   launch "window" : key-sparse attention (sink + block-anchored sliding
//                     window, delta_attention/train/flex_delta.py:59-61) for
//                     every row below s_p, with the delta correction of
//                     delta_attention/llama.py:733-757 fused into the epilogue:
//                     out = sparse + (dense[a] - sparse[a]) for the owning anchor
//                     a.  The sparse output never goes to HBM.  With fuse_delta
//                     (gamma 64, 4 heads per KV group) each job's tile A holds
//                     the job's anchor row and forms dense - sparse for it.
//
// A job is two 128-row query tiles ("A" and "B"); a tile is R rows x G heads of
// one KV group (R = 128 / G), so the whole GQA group shares every K/V tile.
// Three warpgroups (384 threads, launched at REGS_LAUNCH registers each and
// re-split with setmaxnreg: control REGS_CTRL, softmax REGS_SOFTMAX):
//   warp 0       : producer (job fetch and key-tile plan, Q by TMA or cp.async
//                  gather into two Q slots, K and V by TMA into 2-stage rings)
//   warp 1       : TMEM owner and MMA issuer: the warp runs the issue loop and
//                  one elected lane issues every tcgen05.mma and commit
//   warps 2, 3   : idle
//   warps 4..7   : softmax of tile A, one thread per row (TMEM lane); at the end
//                  of a job the same warps read O, hand the accumulator back to
//                  the MMA issuer and store the normalised, corrected rows
//                  (full window tiles through a staging tile and a TMA store)
//   warps 8..11  : softmax (and epilogue) of tile B
// Each query tile has one S buffer in TMEM and the MMA issue order per key tile
// i is PV_A(i), S_A(i+1), PV_B(i), S_B(i+1), so the softmax of one query tile
// overlaps the matrix products of the other.
// TMEM (512 columns): S_A, S_B (128 fp32 columns each; P is written back over
// the first 64 columns of its S buffer as packed bf16 and read by the TS-form
// MMA), then O_A, O_B (head_dim columns each) from column 256.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cmath>
#include <cstddef>
#include <type_traits>

#include "dta_ptx.cuh"
#include "dta_prefill.h"
#include "dta_prefill_jobs.cuh"

namespace dta {

// delta[b, a, h, :] = dense_buf - sparse_buf: bf16 for the windowed launch,
// optionally fp32 for telemetry
__global__ void anchor_delta_kernel(const float* __restrict__ dense, const float* __restrict__ sparse,
                                    __nv_bfloat16* __restrict__ out_bf16, float* __restrict__ out_f32, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(dense)[i];
    const float4 b = reinterpret_cast<const float4*>(sparse)[i];
    const float4 d = make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
    uint2 w;
    w.x = pack_bf16x2(d.x, d.y);
    w.y = pack_bf16x2(d.z, d.w);
    reinterpret_cast<uint2*>(out_bf16)[i] = w;
    if (out_f32) reinterpret_cast<float4*>(out_f32)[i] = d;
  }
}

cudaError_t launch_anchor_delta(const float* dense, const float* sparse, __nv_bfloat16* delta_bf16, float* delta_f32,
                                long long n, cudaStream_t s) {
  const long long n4 = n / 4;
  int blocks = (int)((n4 + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  anchor_delta_kernel<<<blocks, 256, 0, s>>>(dense, sparse, delta_bf16, delta_f32, n4);
  return cudaGetLastError();
}

}  // namespace dta

namespace dta {

constexpr int BM = 128;
constexpr int BN = PREFILL_BN;  // keys per tile
constexpr int NUM_THREADS = 128 + PREFILL_NQ * 128;
constexpr int CTRL_BYTES = 2048;
#ifndef DTA_REGS_CTRL
#define DTA_REGS_CTRL 96
#endif
#ifndef DTA_REGS_SOFTMAX
#define DTA_REGS_SOFTMAX 200
#endif
// registers per thread at launch (one CTA per SM), rounded down to 8
constexpr int REGS_LAUNCH = (65536 / NUM_THREADS) & ~7;
constexpr int REGS_CTRL = DTA_REGS_CTRL, REGS_SOFTMAX = DTA_REGS_SOFTMAX;
static_assert(128 * REGS_CTRL + PREFILL_NQ * 128 * REGS_SOFTMAX <= NUM_THREADS * REGS_LAUNCH,
              "register split exceeds the launch budget");
constexpr int NQ = PREFILL_NQ;

template <int HD>
struct Geo {
  static constexpr int REGIONS = HD / 64;           // 128-byte swizzle atoms along head_dim
  static constexpr int REGION_BYTES = 128 * 128;    // Q: 128 rows x 128 bytes
  static constexpr int TILE_BYTES = REGIONS * REGION_BYTES;  // one 128 x HD bf16 Q tile
  static constexpr int KV_REGION_BYTES = BN * 128;  // K/V: BN rows x 128 bytes
  static constexpr int KV_TILE_BYTES = REGIONS * KV_REGION_BYTES;
#ifndef DTA_K_STAGES
#define DTA_K_STAGES 2
#endif
#ifndef DTA_V_STAGES
#define DTA_V_STAGES 2
#endif
  static constexpr int K_STAGES = DTA_K_STAGES;
  static constexpr int V_STAGES = DTA_V_STAGES;
  static constexpr int Q_OFF = CTRL_BYTES;
  static constexpr int K_OFF = Q_OFF + NQ * TILE_BYTES;  // one Q slot per query tile
  static constexpr int V_OFF = K_OFF + K_STAGES * KV_TILE_BYTES;
  // staging tile of the window launch's TMA-store epilogue (one 128-row bf16 tile)
  static constexpr int STG_OFF = V_OFF + V_STAGES * KV_TILE_BYTES;
  // two staging halves of 128 rows x 128 bytes (64 bf16 columns), one per query tile
  static constexpr int STG_HALF = 128 * 128;
  static constexpr int SMEM_BYTES = STG_OFF + 2 * STG_HALF + 1024;  // + alignment slack
  static constexpr int TMEM_COLS = 512;
  static constexpr int S_COL = 0;    // S of tile q at q * BN
  static constexpr int O_COL = 256;  // O of tile q at 256 + q * 128
};
static_assert(Geo<128>::SMEM_BYTES <= 232448, "shared memory budget");

struct Ctrl {
  uint64_t job_full[2], job_empty[2];
  uint64_t q_full[NQ], q_empty[NQ];
  uint64_t k_full[4], k_empty[4], v_full[4], v_empty[4];
  // p_full[2 * q + h]: half h of P_q (keys [h * BN/2, (h+1) * BN/2))
  uint64_t s_full[NQ], p_full[NQ * 2], o_full[NQ], o_empty[NQ];
  uint64_t stg_full[NQ];    // tile q's rows are in its staging half (4 warps)
  uint64_t stg_free[NQ];    // the last TMA store from tile q's staging half has read it
  uint64_t drain;
  uint64_t stall;           // test hook: a barrier that nothing completes
  uint64_t delta_ready;     // pair delta: tile A wrote this job's anchor rows (4 warps)
  uint64_t delta_free;      // pair delta: tile B read them (4 warps)
  alignas(16) uint32_t dslot[4][64];  // pair delta: bf16 (dense - sparse) row of each head's anchor (read as uint4)
  int job[2][8];
  Plan plan[2];             // key-tile plan of job[slot], computed once by the producer
  uint32_t tmem_base;
  int abort_flag;
  // fused delta across warps: anchor rows formed so far by this CTA's warps
  // (one count per forming warp and anchor period; only ever grows)
  int delta_count;
  // split dense jobs: per softmax warp, (chunk | active chunks << 16) of its
  // current job, or -1; kept here so it is not held in registers across the
  // key-tile loop
  int split_word[4 * NQ];
};
static_assert(offsetof(Ctrl, dslot) % 16 == 0, "dslot is read with 16-byte loads");
static_assert(sizeof(Ctrl) <= CTRL_BYTES, "control block too large");

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// bits c >= lo of a 32-bit column word (all for lo <= 0, none for lo >= 32)
__device__ __forceinline__ uint32_t bits_from(int lo) {
  return lo <= 0 ? 0xffffffffu : (lo >= 32 ? 0u : (0xffffffffu << lo));
}

// LK (a Launch) and FM (a FuseMode, windowed launch) are compile-time
// parameters: the windowed kernel carries no row-list, split-K or dense-row
// code and the rows kernel no staging, TMA-store or fused-delta code, and each
// fused-delta arrangement has its own windowed kernel, so every variant is
// register-allocated for its own work.
template <int HD, int LK, int FM>
__global__ void __launch_bounds__(NUM_THREADS, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
  using G = Geo<HD>;
  constexpr bool WIN = (LK == LAUNCH_WINDOW);
  constexpr bool FUSE = WIN && FM != FUSE_NONE;  // the windowed launch forms the delta
  constexpr bool PAIR = WIN && FM == FUSE_PAIR;  // ... tile A for tile B through shared memory
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
  // (the budget is read from the launch parameters, not held in a register)
  const WaitCtx wc{abort_flag, err, p.wait_cycles};

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(BAR(job_full[0]) + 8 * i, 1);
      mbar_init(BAR(job_empty[0]) + 8 * i, 1 + 4 * NQ);  // MMA thread + softmax warps
    }
    for (int i = 0; i < NQ; ++i) {
      mbar_init(BAR(q_full[0]) + 8 * i, 1);
      mbar_init(BAR(q_empty[0]) + 8 * i, 1);
    }
    for (int i = 0; i < G::K_STAGES; ++i) {
      mbar_init(BAR(k_full[0]) + 8 * i, 1);
      mbar_init(BAR(k_empty[0]) + 8 * i, 1);
    }
    for (int i = 0; i < G::V_STAGES; ++i) {
      mbar_init(BAR(v_full[0]) + 8 * i, 1);
      mbar_init(BAR(v_empty[0]) + 8 * i, 1);
    }
    for (int q = 0; q < NQ; ++q) {
      mbar_init(BAR(s_full[0]) + 8 * q, 1);
      mbar_init(BAR(p_full[0]) + 8 * (2 * q), 4);
      mbar_init(BAR(p_full[0]) + 8 * (2 * q + 1), 4);
      mbar_init(BAR(o_full[0]) + 8 * q, 1);
      mbar_init(BAR(o_empty[0]) + 8 * q, 4);  // softmax warps of tile q, after reading O
    }
    for (int q = 0; q < NQ; ++q) {
      mbar_init(BAR(stg_full[0]) + 8 * q, 4);
      mbar_init(BAR(stg_free[0]) + 8 * q, 1);
    }
    mbar_init(BAR(drain), 1);
    mbar_init(BAR(stall), 1);
    mbar_init(BAR(delta_ready), 4);
    mbar_init(BAR(delta_free), 4);
    ctrl->abort_flag = 0;
    ctrl->delta_count = 0;
    mbar_init_fence();
  }
  // rows launch: a windowed launch queued behind this one may start its CTAs
  // as this grid's CTAs run out of jobs and exit
  if (!WIN && threadIdx.x == 0) grid_dependents_launch();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    if (WIN) tma_prefetch_desc(&p.tm_q);
    if (WIN && p.tma_out) tma_prefetch_desc(&p.tm_out);
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

  if (warp < 4) {
  regs_release<REGS_CTRL>();
  if (warp == 0) {
    // ======================= producer =======================
    int n = 0;                // K/V tiles issued so far (ring position)
    int nk = 0, nv = 0;       // K / V tile loads issued (for the drain on abort)
    int q_fills[NQ] = {0, 0};  // Q loads issued per slot (tile q uses slot q)
    int fetched = 0;          // window launch: jobs taken from this CTA's static stride
    bool ok = true;
    if (p.test_stall) {
      // test hook: wait for a barrier phase that never completes, so this
      // wait runs out after the budget and the CTA takes the abort path
      ok = mbar_wait_warp(BAR(stall), 0, wc, KERR_TIMEOUT_PRODUCER);
    }
    for (int it = 0; ok; ++it) {
      const int slot = it & 1;
      // the plan goes out with the job: the consumers would otherwise each
      // run make_plan, cold code on their critical path at every job change.
      // Chunk slots past a short row tile's chunks are empty and skipped here.
      Job J;
      Plan P{};
      for (;;) {
        int j;
        if constexpr (WIN) {
          // static stride over groups of win_group consecutive jobs (one
          // anchor period when it spans several jobs, so the job forming its
          // delta runs first, on this CTA)
          const int f = fetched++;
          j = (FM != FUSE_GENERAL || p.win_group == 1)
                  ? blockIdx.x + f * gridDim.x
                  : (blockIdx.x + (f / p.win_group) * gridDim.x) * p.win_group + f % p.win_group;
        } else {
          int jj = 0;
          if (lane == 0) jj = atomicAdd(p.counter, 1);
          j = __shfl_sync(0xffffffffu, jj, 0);
        }
        J = decode_job(p, j);
        if (J.kind == JOB_END) break;
        P = make_plan(p, J);
        if (P.n_tiles > 0) break;
      }
      if (!mbar_wait_warp(BAR(job_empty[0]) + 8 * slot, ((it >> 1) & 1) ^ 1, wc,
                          KERR_TIMEOUT_PRODUCER))
        break;
      if (lane == 0) {
        int* dst = ctrl->job[slot];
        dst[0] = J.kind; dst[1] = J.b; dst[2] = J.g; dst[3] = J.start; dst[4] = J.count; dst[5] = J.chunk;
        if (J.kind != JOB_END) ctrl->plan[slot] = P;
        mbar_arrive(BAR(job_full[0]) + 8 * slot);  // release: job and plan are visible to the waiters
      }
      if (J.kind == JOB_END) break;
      // Q slots (mirrored by the MMA issuer): tile q keeps slot q, which the
      // previous job's tile q frees at its last S.  Loads go in the order
      // Q_B, K0, V0, Q_A, K1, V1, ...  (q is a compile-time constant at
      // every call, so the per-slot state stays in registers)
      auto load_q = [&](auto qc) -> bool {
        constexpr int q = decltype(qc)::value, qs = q;
        if (P.tiles_t[q] == 0) return true;
        const uint32_t qbuf = q_u32 + (uint32_t)qs * G::TILE_BYTES;
        if (!mbar_wait_warp(BAR(q_empty[0]) + 8 * qs, (q_fills[qs] & 1) ^ 1, wc, KERR_TIMEOUT_PRODUCER))
          return false;
        ++q_fills[qs];
        if constexpr (WIN) {
          if (lane == 0) {
            mbar_arrive_expect_tx(BAR(q_full[0]) + 8 * qs, G::TILE_BYTES);
            for (int r = 0; r < G::REGIONS; ++r)
              tma_load_4d(qbuf + r * G::REGION_BYTES, &p.tm_q, BAR(q_full[0]) + 8 * qs, r * 64,
                          J.start + q * p.R, J.g * p.G, J.b);
          }
        } else {
          // gather R list rows x G heads with cp.async into the 128-byte-
          // swizzled K-major layout the MMA expects
          constexpr int CH = HD / 8;  // 16-byte chunks per row
          const __nv_bfloat16* qb = p.q + (long long)J.b * p.q_sb;
          const int r_shift = __ffs(p.R) - 1;  // R = 128 / G is a power of two
          for (int c = lane; c < BM * CH; c += 32) {
            const int m = c / CH, cc = c - (c / CH) * CH;
            const int hh = m >> r_shift, rr = m & (p.R - 1);
            const int li = q * p.R + rr;
            const bool valid = li < J.count;
            const int row = valid ? clamp_row(p, list_q_row(p, J.start + li), p.seq_q) : 0;
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
        return true;
      };
      if (!load_q(std::integral_constant<int, 1>{})) break;
      // ---- K and V tiles (Q_A after the first pair) ----
      for (int i = 0; i < P.n_tiles; ++i, ++n) {
        const int st = n % G::K_STAGES, sv = n % G::V_STAGES;
        const uint32_t ph = (uint32_t)((n / G::K_STAGES) & 1), phv = (uint32_t)((n / G::V_STAGES) & 1);
        const int ks = tile_key_start(P, i);
        if (!mbar_wait_warp(BAR(k_empty[0]) + 8 * st, ph ^ 1, wc, KERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t kdst = k_u32 + (uint32_t)st * G::KV_TILE_BYTES;
          mbar_arrive_expect_tx(BAR(k_full[0]) + 8 * st, G::KV_TILE_BYTES);
          for (int r = 0; r < G::REGIONS; ++r)
            tma_load_4d(kdst + r * G::KV_REGION_BYTES, &p.tm_k, BAR(k_full[0]) + 8 * st, r * 64, ks, J.g, J.b);
        }
        nk = n + 1;
        if (!mbar_wait_warp(BAR(v_empty[0]) + 8 * sv, phv ^ 1, wc, KERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t vdst = v_u32 + (uint32_t)sv * G::KV_TILE_BYTES;
          mbar_arrive_expect_tx(BAR(v_full[0]) + 8 * sv, G::KV_TILE_BYTES);
          for (int r = 0; r < G::REGIONS; ++r)
            tma_load_4d(vdst + r * G::KV_REGION_BYTES, &p.tm_v, BAR(v_full[0]) + 8 * sv, r * 64, ks, J.g, J.b);
        }
        nv = n + 1;
        if (i == 0 && !load_q(std::integral_constant<int, 0>{})) {
          ok = false;
          break;
        }
      }
    }
    // On abort, let in-flight TMA loads land before the CTA can exit: at most
    // the last K_STAGES K loads, V_STAGES V loads and one Q load per slot can
    // still be in flight (each load waited for its stage to be consumed).
    if (*abort_flag && lane == 0) {
      auto drain = [](uint32_t bar, uint32_t parity) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar, parity))
          if (clock64() - t0 > kWaitTimeoutCycles) break;
      };
      for (int m = max(0, nk - G::K_STAGES); m < nk; ++m)
        drain(BAR(k_full[0]) + 8 * (m % G::K_STAGES), (uint32_t)((m / G::K_STAGES) & 1));
      for (int m = max(0, nv - G::V_STAGES); m < nv; ++m)
        drain(BAR(v_full[0]) + 8 * (m % G::V_STAGES), (uint32_t)((m / G::V_STAGES) & 1));
      if (q_fills[0] > 0) drain(BAR(q_full[0]), (uint32_t)((q_fills[0] - 1) & 1));
      if (q_fills[1] > 0) drain(BAR(q_full[0]) + 8, (uint32_t)((q_fills[1] - 1) & 1));
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    // The whole warp runs the issue loop (warp-uniform waits, descriptors and
    // counters) and one elected lane issues each batch of tcgen05.mma and
    // commits.  Per-query-tile state is indexed only by compile-time tile
    // numbers (the lambdas take std::integral_constant), so it stays in
    // registers: this warp sits on the S -> softmax -> P -> PV chain and must
    // react to a released P within a few cycles.
    {
      using QA = std::integral_constant<int, 0>;
      using QB = std::integral_constant<int, 1>;
      constexpr uint32_t IDESC_QK = idesc_bf16_f32(128, BN, 0);
      constexpr uint32_t IDESC_PV = idesc_bf16_f32(128, HD, 1);
      // base descriptors: Q slot 0 / K stage 0 (K-major), V stage 0 (MN-major)
      const uint64_t qdesc0 = smem_desc_sw128(q_u32, 16, 1024);
      const uint64_t kdesc0 = smem_desc_sw128(k_u32, 16, 1024);
      const uint64_t vdesc0 = smem_desc_sw128(v_u32, G::KV_REGION_BYTES, 1024);
      int n = 0;                   // K/V tiles consumed so far (ring position)
      int q_uses[NQ] = {0, 0};     // Q loads consumed per slot (tile q uses slot q)
      int cnt_pv[NQ] = {0, 0};     // PV products issued per query tile
      int jobs_t[NQ] = {0, 0};     // jobs in which query tile q was active
      bool aborted = false;
      for (int it = 0; !aborted; ++it) {
        const int slot = it & 1;
        if (!mbar_poll(BAR(job_full[0]) + 8 * slot, (it >> 1) & 1, wc, KERR_TIMEOUT_MMA)) break;
        Job J;
        {
          const volatile int* src = ctrl->job[slot];
          J.kind = src[0]; J.b = src[1]; J.g = src[2]; J.start = src[3]; J.count = src[4];
        }
        const Plan P = ctrl->plan[slot];  // read before the slot is released
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR(job_empty[0]) + 8 * slot);
        if (J.kind == JOB_END) break;
        const int tiles[NQ] = {P.tiles_t[0], P.tiles_t[1]};
        const int n0 = n;  // ring position of this job's key tile 0
        // S_q(i) = Q_q . K_i^T.  K_i is released by the last query tile that uses it.
        auto issue_s = [&](auto qc, int i) -> bool {
          constexpr int q = decltype(qc)::value;
          const int m = n0 + i, st = m % G::K_STAGES;
          if (i == 0) {
            if (!mbar_poll(BAR(q_full[0]) + 8 * q, q_uses[q] & 1, wc, KERR_TIMEOUT_MMA)) return false;
            ++q_uses[q];
          }
          if (q == 0 || i >= tiles[0]) {  // first user of K_i waits for it
            if (!mbar_poll(BAR(k_full[0]) + 8 * st, (m / G::K_STAGES) & 1, wc, KERR_TIMEOUT_MMA))
              return false;
          }
          tc_fence_after();
          const uint32_t tS = tmem + G::S_COL + q * BN;
          // descriptors differ only in the 14-bit start-address field, which
          // never carries out (shared memory < 256 KB), so offsets are plain adds
          const uint64_t qd = qdesc0 + (((uint32_t)q * G::TILE_BYTES) >> 4);
          const uint64_t kd = kdesc0 + (((uint32_t)st * G::KV_TILE_BYTES) >> 4);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint32_t qoff = ((kk >> 2) * G::REGION_BYTES + (kk & 3) * 32) >> 4;
              const uint32_t koff = ((kk >> 2) * G::KV_REGION_BYTES + (kk & 3) * 32) >> 4;
              umma_ss(tS, qd + qoff, kd + koff, IDESC_QK, kk > 0 ? 1u : 0u);
            }
            umma_commit(BAR(s_full[0]) + 8 * q);
            if (q == NQ - 1 || i >= tiles[NQ - 1]) umma_commit(BAR(k_empty[0]) + 8 * st);
            if (i == tiles[q] - 1) umma_commit(BAR(q_empty[0]) + 8 * q);
          }
          __syncwarp();
          return true;
        };
        // O_q += P_q(i) . V_i, in two halves of the key tile: the first half
        // of P is released while the softmax still computes the second
        auto issue_pv = [&](auto qc, int i) -> bool {
          constexpr int q = decltype(qc)::value;
          const int m = n0 + i, st = m % G::V_STAGES;
          const uint32_t pbar = BAR(p_full[0]) + 8 * (2 * q);
          const uint32_t pph = (uint32_t)(cnt_pv[q] & 1);
          if (!mbar_poll(pbar, pph, wc, KERR_TIMEOUT_MMA)) return false;
          if (i == 0 && jobs_t[q] > 0) {
            if (!mbar_poll(BAR(o_empty[0]) + 8 * q, (jobs_t[q] - 1) & 1, wc, KERR_TIMEOUT_MMA))
              return false;
          }
          if (q == 0 || i >= tiles[0]) {  // first user of V_i waits for it
            if (!mbar_poll(BAR(v_full[0]) + 8 * st, (m / G::V_STAGES) & 1, wc, KERR_TIMEOUT_MMA))
              return false;
          }
          tc_fence_after();
          const uint32_t tP = tmem + G::S_COL + q * BN;
          const uint32_t tO = tmem + G::O_COL + q * 128;
          const uint64_t vd = vdesc0 + (((uint32_t)st * G::KV_TILE_BYTES) >> 4);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < BN / 32; ++kk)
              umma_ts(tO, tP + kk * 8, vd + ((kk * 2048) >> 4), IDESC_PV, (i == 0 && kk == 0) ? 0u : 1u);
          }
          __syncwarp();
          if (!mbar_poll(pbar + 8, pph, wc, KERR_TIMEOUT_MMA)) return false;
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int kk = BN / 32; kk < BN / 16; ++kk) umma_ts(tO, tP + kk * 8, vd + ((kk * 2048) >> 4), IDESC_PV, 1u);
            // O of this job is final after its last PV: the epilogue's signal.  (The
            // softmax needs no per-PV signal: the S_q(i + 1) commit covers PV_q(i).)
            if (i == tiles[q] - 1) umma_commit(BAR(o_full[0]) + 8 * q);
            if (q == NQ - 1 || i >= tiles[NQ - 1]) umma_commit(BAR(v_empty[0]) + 8 * st);
          }
          __syncwarp();
          ++cnt_pv[q];
          return true;
        };
        // prologue: S of key tile 0 for every active query tile; then per key
        // tile i: PV_A(i), S_A(i+1), PV_B(i), S_B(i+1)
        if ((tiles[0] > 0 && !issue_s(QA{}, 0)) || (tiles[1] > 0 && !issue_s(QB{}, 0))) break;
        for (int i = 0; i < P.n_tiles; ++i) {
          if (i < tiles[0] && (!issue_pv(QA{}, i) || (i + 1 < tiles[0] && !issue_s(QA{}, i + 1)))) {
            aborted = true;
            break;
          }
          if (i < tiles[1] && (!issue_pv(QB{}, i) || (i + 1 < tiles[1] && !issue_s(QB{}, i + 1)))) {
            aborted = true;
            break;
          }
        }
        if (aborted) break;
        for (int q = 0; q < NQ; ++q)
          if (tiles[q] > 0) ++jobs_t[q];
        n += P.n_tiles;
      }
      // drain: every issued tcgen05 op completes before TMEM is released
      // (tcgen05 ops complete in issue order, and the elected lanes of one
      // warp issue in program order)
      __syncwarp();
      if (elect_one()) umma_commit(BAR(drain));
      __syncwarp();
      const long long t0 = clock64();
      while (!mbar_try_wait(BAR(drain), 0)) {
        if (clock64() - t0 > kWaitTimeoutCycles) {
          atomicCAS(err, 0, KERR_TIMEOUT_DRAIN);
          break;
        }
      }
    }
  }
  } else if (warp < 4 + 4 * NQ) {
    regs_acquire<REGS_SOFTMAX>();
    // ======================= softmax =======================
    const int q = (warp - 4) >> 2;        // query tile of this warpgroup
    const int quarter = warp & 3;         // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;    // row of this thread inside its query tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int hh = r >> (__ffs(p.R) - 1);  // head of this row inside the KV group (R = 128 / G, a power of two)
    const int rr = r & (p.R - 1);
    const uint32_t tS = tmem + lane_off + G::S_COL + q * BN;
    const uint32_t tO = tmem + lane_off + G::O_COL + q * 128;
    const float sl2 = p.scale_log2;
    int cnt = 0;        // S tiles consumed by this warpgroup (= PVs of its query tile)
    int jobs_done = 0;  // jobs in which this query tile was active
    int st_rounds = 0;  // 64-column TMA-store rounds through this tile's staging half
    bool st_pending = false;  // (leader) the last round's store has not been waited for
    bool dep_done = false;  // the rows launch's output may be read (windowed launch)
    int periods = 0;    // fused delta across warps: anchor periods this tile has entered
    int f_writes = 0;   // pair delta: anchor rows published by tile A so far
    int f_reads = 0;    // pair delta: of those, read by tile B
    for (int it = 0;; ++it) {
      const int slot = it & 1;
      if (!mbar_wait_warp(BAR(job_full[0]) + 8 * slot, (it >> 1) & 1, wc, KERR_TIMEOUT_SOFTMAX)) break;
      Job J;
      {
        const volatile int* src = ctrl->job[slot];
        J.kind = src[0]; J.b = src[1]; J.g = src[2]; J.start = src[3]; J.count = src[4];
      }
      const Plan P = ctrl->plan[slot];  // read before the slot is released
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(BAR(job_empty[0]) + 8 * slot);
        ctrl->split_word[warp - 4] =
            (!WIN && J.kind == JOB_DENSE_ROWS && P.n_chunks > 1) ? (P.chunk | ((q ? P.act_t[1] : P.act_t[0]) << 16))
                                                                 : -1;
      }
      if (J.kind == JOB_END) break;
      // this warpgroup's tile: selects, not a dynamic index, so the plan stays in registers
      const int T = q ? P.tiles_t[1] : P.tiles_t[0];
      // Window-launch tiles whose 128 rows all lie below row_end leave through
      // this tile's staging half and TMA stores (recompute mode skips anchor
      // rows, so it stores row by row).
      const bool use_stg = WIN && p.tma_out && p.mode != 1 && T > 0 &&
                           J.start + (q + 1) * p.R <= p.row_end;
      // fused delta (windowed launch, uniform anchors): the warp holding an
      // anchor row forms dense - sparse for it in its epilogue; with anchors
      // at most R apart every warp forms its own rows' anchors, otherwise the
      // first job of each anchor period forms them in tile A and the other
      // tiles of the period wait for them (delta_count)
      constexpr bool fuse = FUSE;
      // pair delta (gamma = 64 with 4 heads per group: a 64-row job starts at
      // its anchor, which is row 0 of tile A for every head): tile A hands each
      // head's delta row to tile B through shared memory.  Both warpgroups
      // count every job.
      constexpr bool pair = PAIR;
      const int f_writes_prev = f_writes, f_reads_prev = f_reads;
      if (pair && P.tiles_t[0] > 0) ++f_writes;
      if (pair && P.tiles_t[0] > 0 && P.tiles_t[1] > 0) ++f_reads;
      if (fuse && !pair && p.delta_cross && J.start == fast_div(J.start, p.gamma_mul, p.gamma_sh) * p.gamma)
        ++periods;
      if (T == 0) continue;  // this query tile is empty in this job
      const int li = q * p.R + rr;  // job-local row
      const bool row_valid = li < J.count;
      const int qpos = row_valid ? job_row_pos(p, J, li) : (q ? P.qmax_t[1] : P.qmax_t[0]);
      const bool sparse_kind = WIN || (J.kind != JOB_DENSE_ROWS);
      const int lo_q = sparse_kind ? block_window_lo(p, qpos) : 0;
      const int sink_q = sparse_kind ? p.sink : 0x7fffffff;
      const int qmin_t = q ? P.qmin_t[1] : P.qmin_t[0];
      // the owning anchor's delta row (window launch, delta mode), pulled into
      // L1 now for the epilogue at the end of the job
      const __nv_bfloat16* dlt = nullptr;
      const long long anchor_row = ((long long)J.b * p.n_anchor + anchor_of(p, qpos)) * p.H + J.g * p.G + hh;
      // (prefetches of the rows launch's output only once it has completed:
      // before that, under a programmatic dependent launch, it may be unwritten)
      if (pair) {
        // tile A: its head's anchor dense row (fp32, written by the rows launch)
        // goes to L2 now; each lane loads 4 columns of it at the end of the job
        if (q == 0 && lane < HD * 4 / 128 && dep_done)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(p.dense_buf + anchor_row * HD) + lane * 128));
      } else if (fuse) {
        // an anchor row's dense row (fp32, written by the rows launch) goes to
        // L2 now; the warp reads it at the end of the job to form the delta
        // (anchor rows: recomputed in the epilogue rather than held across the key loop)
        if (row_valid && qpos == fast_div(qpos, p.gamma_mul, p.gamma_sh) * p.gamma && dep_done) {
#pragma unroll
          for (int c = 0; c < HD * 4 / 128; ++c)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(p.dense_buf + anchor_row * HD) + c * 128));
        }
      } else if (WIN && p.mode == 0 && p.delta_buf) {
        dlt = p.delta_buf + anchor_row * HD;
        if (dep_done)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const char*>(dlt) + (lane & (HD * 2 / 128 - 1)) * 128));
      }
      const int lo_max_t = q ? P.lo_max_t[1] : P.lo_max_t[0];

      float m_run = -INFINITY, l_run = 0.f;
      bool aborted = false;
      for (int i = 0; i < T; ++i, ++cnt) {
        if (!mbar_wait_warp(BAR(s_full[0]) + 8 * q, cnt & 1, wc,
                            KERR_TIMEOUT_SOFTMAX)) {
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
        // column window of this row: valid iff A <= c <= Bq and not X <= c < Y,
        // as one validity bit per column (32 per word), then one bit test and
        // one select per element
        const int mA = seg_lo - ks;
        const int mB = min(seg_hi - 1, qpos) - ks;
        const int mX = sink_q - ks;
        const int mY = lo_q - ks;
        auto mask_word = [&](int w) {
          const int o = 32 * w;
          const uint32_t m = bits_from(mA - o) & ~bits_from(mB + 1 - o) & ~(bits_from(mX - o) & ~bits_from(mY - o));
#pragma unroll
          for (int e = 0; e < 32; ++e) x[o + e] = ((m >> e) & 1u) ? x[o + e] : -INFINITY;
        };
        if (!full) {
#pragma unroll
          for (int w = 0; w < BN / 32; ++w) mask_word(w);
        }
        // row max: 8 independent chains of three-input maxima (scaled, log2 domain)
        auto row_max = [&]() -> float {
          float mk[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float m = fmax3(x[k], x[k + 8], x[k + 16]);
#pragma unroll
            for (int j = 3; j + 1 < BN / 8; j += 2) m = fmax3(m, x[k + 8 * j], x[k + 8 * (j + 1)]);
            mk[k] = fmaxf(m, x[k + BN - 8]);
          }
          return fmax3(fmax3(mk[0], mk[1], mk[2]), fmax3(mk[3], mk[4], mk[5]), fmaxf(mk[6], mk[7])) * sl2;
        };
        // The running max is kept unless a tile raises it by more than 2^8
        // (exact: O and l always share the reference max; P stays <= 256).  So
        // after the first tile of a job the exponentials of the first 32 keys
        // start from the running max while this tile's max is computed beside
        // them; in the rare case that it grew too much, they are recomputed.
        if (i == 0) m_run = row_max();
        // P = exp2(S * scale - m): scale/shift and row sums on packed fp32 pairs
        const uint64_t sc2 = f2_pack(sl2, sl2);
        uint64_t ls2[4];
        auto exp_chunk = [&](int c, uint32_t (&pk)[16], uint64_t nm2) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float a0, a1, p0, p1;
            f2_unpack(f2_fma(f2_pack(x[c * 32 + 2 * e], x[c * 32 + 2 * e + 1]), sc2, nm2), a0, a1);
            p0 = fast_exp2(a0);
            p1 = fast_exp2(a1);
            ls2[e & 3] = f2_add(ls2[e & 3], f2_pack(p0, p1));
            pk[e] = pack_bf16x2(p0, p1);
          }
        };
        auto neg_m = [](float m) { const float u = (m == -INFINITY) ? 0.f : m; return f2_pack(-u, -u); };
        uint32_t pk0[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) ls2[k] = f2_pack(0.f, 0.f);
        exp_chunk(0, pk0, neg_m(m_run));
        const float mt = row_max();
        const bool need = (i > 0) && (mt > m_run + 8.0f);
        const bool any_need = __any_sync(0xffffffffu, need);
        const float m_old = m_run;
        if (any_need) {
          // rare: the max grew by more than 2^8 for some row of the warp.  Those
          // rows redo the first 32 keys with the new max (and rescale O below)
          const float m_new = need ? mt : m_run;
          // S is still in TMEM (P has not been written): reload the first 32 keys
          tmem_ld32f(tS, x);
          tmem_wait_ld();
          if (!full) mask_word(0);
#pragma unroll
          for (int k = 0; k < 4; ++k) ls2[k] = f2_pack(0.f, 0.f);
          exp_chunk(0, pk0, neg_m(m_new));
          m_run = m_new;
        }
        const uint32_t pbar = BAR(p_full[0]) + 8 * (2 * q);
        __syncwarp();  // converge before the warp-collective TMEM stores
        tmem_st16(tS, pk0);
        {
          uint32_t pk1[16];
          exp_chunk(1, pk1, neg_m(m_run));
          tmem_st16(tS + 16, pk1);
        }
        if (any_need) {
          // O rescale for rows whose max moved (here, with half of the S row
          // dead, to keep registers low).  The S_q(i) commit covers every
          // earlier MMA, so PV(i-1) is complete; the TMEM round trip is
          // warp-collective and other rows scale by 1.
          const float alpha = !need ? 1.f : ((m_old == -INFINITY) ? 0.f : fast_exp2(m_old - m_run));
#pragma unroll
          for (int c2 = 0; c2 < HD / 32; ++c2) {
            uint32_t o[32];
            tmem_ld32(tO + c2 * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + c2 * 32, o);
          }
          if (need) l_run *= alpha;
        }
        // the first half of P (keys [0, BN/2)) is in TMEM: release it
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pbar);
#pragma unroll
        for (int c = BN / 64; c < BN / 32; ++c) {
          uint32_t pk[16];
          exp_chunk(c, pk, neg_m(m_run));
          tmem_st16(tS + c * 16, pk);
        }
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
      // ---- epilogue of this tile: O / l (+ delta) to global memory ----
      // The destination and the delta row do not depend on O: they are set up
      // while the last PV runs.  O is read into registers in one batch and
      // released at once (the next job's first PV of this tile waits for it),
      // then normalised and stored.
      const int h = J.g * p.G + hh;
      const int gli = J.start + li;  // list index (row jobs)
      bool store = row_valid;
      int mode_out = 0;  // 0: bf16 to out, 1: fp32 to dense_buf, 2: fp32 to sparse_buf
      long long out_row = 0;
      if constexpr (WIN) {
        out_row = qpos;
        if (store && p.mode == 1) {
          store = !is_anchor_row(p, qpos);
        }
      } else if (J.kind == JOB_DENSE_ROWS) {
        if (gli < p.direct_from) {
          mode_out = 1;
        } else {
          out_row = !row_valid ? 0 : (p.out_by_list ? gli : list_q_row(p, gli));
          if (out_row < 0 || out_row >= p.out_rows) {  // a bad explicit anchor: flagged, not stored
            if (store) atomicCAS(p.error, 0, KERR_BAD_ROW);
            store = false;
          }
        }
      } else {
        mode_out = 2;
      }
      // 1/l to ~2 ulp (__fdividef): far below the bf16 rounding of the output
      const float inv_l = (l_run > 0.f) ? __fdividef(1.f, l_run) : 0.f;
      // the windowed row's base-2 log-sum-exp, kept by the training forward
      if (WIN && p.lse_sparse && row_valid)
        p.lse_sparse[((long long)J.b * p.H + h) * p.seq_q + qpos] = (l_run > 0.f) ? m_run + __log2f(l_run) : -INFINITY;
      if (WIN && !dep_done) {
        // the rows launch (the grid this one may overlap) has completed and its
        // writes are visible before the first read of its output.  Its output
        // (the dense rows) is read through L2 only (ld.global.cg): this grid
        // started while that one ran, so neither the non-coherent read-only
        // path nor L1 is guaranteed to hold current copies of it.
        grid_dependency_wait();
        dep_done = true;
      }
      // fused delta: the anchor rows among this warp's rows, and this lane's 4
      // columns of the dense row of the warp's first anchor (loaded while the
      // last PV runs)
      uint32_t anchor_mask = 0;
      float4 dn_first = make_float4(0.f, 0.f, 0.f, 0.f);
      if (pair) {
        // tile A: lane 0 of every warp holds its head's anchor row
        if (q == 0) dn_first = __ldcg(reinterpret_cast<const float4*>(p.dense_buf + anchor_row * HD) + (lane & (HD / 4 - 1)));
      } else if (fuse) {
        anchor_mask = __ballot_sync(0xffffffffu, row_valid && qpos == fast_div(qpos, p.gamma_mul, p.gamma_sh) * p.gamma);
        if (anchor_mask) {
          const long long arow0 = __shfl_sync(0xffffffffu, anchor_row, __ffs(anchor_mask) - 1);
          dn_first = __ldcg(reinterpret_cast<const float4*>(p.dense_buf + arow0 * HD) + (lane & (HD / 4 - 1)));
        } else if (p.delta_cross) {
          // a consumer tile: its rows' delta lines into L1 early (a prefetch is
          // only a hint; the read after the delta_count wait is what is ordered)
#pragma unroll
          for (int c = 0; c < HD * 2 / 128; ++c)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const char*>(p.delta_buf + anchor_row * HD) + c * 128));
        }
      }
      // o_full[q] completes once per job of this tile (after its last PV); the
      // next job's first PV waits for o_empty[q], so phases cannot run ahead
      if (!mbar_wait_warp(BAR(o_full[0]) + 8 * q, jobs_done & 1, wc, KERR_TIMEOUT_SOFTMAX)) break;
      tc_fence_after();
      float o[HD];
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) tmem_ld32f(tO + c * 32, o + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR(o_empty[0]) + 8 * q);
      ++jobs_done;
      if constexpr (!WIN) {
      __syncwarp();
      const int split_word = *reinterpret_cast<volatile int*>(&ctrl->split_word[warp - 4]);
      if (split_word >= 0) {
        // ---- split dense job: store this chunk's partial (O / l and the
        // log2-sum-exp of every row); the chunk that finishes last merges all
        // of them and stores the rows ----
        const int r_shift = __ffs(p.R) - 1;
        const long long tile_id = (long long)(J.b * p.Hkv + J.g) * p.n_dense_tiles + (J.start >> (r_shift + 1));
        const int act = split_word >> 16;
        const int chunk = split_word & 0xffff;
        auto slot_of = [&](int k) { return ((tile_id * p.split_cmax + k) * NQ + q) * 128; };
        const float lse = (l_run > 0.f) ? m_run + __log2f(l_run) : -INFINITY;
        {
          float4* po = reinterpret_cast<float4*>(p.part_o) + slot_of(chunk) * (HD / 4) + r;
#pragma unroll
          for (int c4 = 0; c4 < HD / 4; ++c4)
            po[c4 * 128] = make_float4(o[4 * c4] * inv_l, o[4 * c4 + 1] * inv_l, o[4 * c4 + 2] * inv_l,
                                       o[4 * c4 + 3] * inv_l);
          p.part_lse[slot_of(chunk) + r] = lse;
        }
        // Each warp counts its own 32 rows' chunks (no barrier across the
        // warpgroup, whose warps may leave the job loop independently on an
        // abort): every lane's partial is visible device-wide before lane 0
        // moves the count.
        __threadfence();
        __syncwarp();
        int done = 0;
        if (lane == 0) done = atomicAdd(p.part_cnt + (tile_id * NQ + q) * 4 + quarter, 1);
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done != act - 1) continue;  // another chunk merges these rows
        __threadfence();
        // Last chunk: log-sum-exp merge of the tile's active chunks, read back
        // from L2 (bypassing L1) 32 columns at a time, so this thread's own O
        // is no longer needed in registers; the rows are stored from here.
        // max and weight sum in one online pass, four loads in flight
        float M = -INFINITY, wsum = 0.f;
        for (int k0 = 0; k0 < act; k0 += 4) {
          float l4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) l4[u] = (k0 + u < act) ? __ldcg(p.part_lse + slot_of(k0 + u) + r) : -INFINITY;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (l4[u] == -INFINITY) continue;
            if (l4[u] > M) {
              wsum = (M == -INFINITY) ? 1.f : fmaf(wsum, fast_exp2(M - l4[u]), 1.f);
              M = l4[u];
            } else {
              wsum += fast_exp2(l4[u] - M);
            }
          }
        }
        const float inv_w = (wsum > 0.f) ? __fdividef(1.f, wsum) : 0.f;
        if (p.lse_dense && row_valid && J.kind == JOB_DENSE_ROWS)
          p.lse_dense[((long long)J.b * p.H + h) * p.n_sel + gli] = (wsum > 0.f) ? M + __log2f(wsum) : -INFINITY;
        __nv_bfloat16* dbf = (store && mode_out == 0)
                                 ? p.out + (((long long)J.b * p.out_rows + out_row) * p.H + h) * HD
                                 : nullptr;
        float* dfl = (store && mode_out == 1) ? p.dense_buf + (((long long)J.b * p.n_anchor + gli) * p.H + h) * HD
                                              : nullptr;
        // weighted sum, 32 columns at a time, four chunks' loads in flight
#pragma unroll 1
        for (int cb = 0; cb < HD / 32; ++cb) {
          float acc[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[e] = 0.f;
          for (int k0 = 0; k0 < act; k0 += 4) {
            float w4[4];
            float4 v4[4][8];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int k = (k0 + u < act) ? k0 + u : k0;  // past the end: reload chunk k0, weight 0
              w4[u] = __ldcg(p.part_lse + slot_of(k) + r);
              const float4* pk = reinterpret_cast<const float4*>(p.part_o) + slot_of(k) * (HD / 4) + cb * 8 * 128 + r;
#pragma unroll
              for (int e = 0; e < 8; ++e) v4[u][e] = __ldcg(pk + e * 128);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float w = (k0 + u >= act || w4[u] == -INFINITY) ? 0.f : fast_exp2(w4[u] - M) * inv_w;
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                acc[4 * e] = fmaf(w, v4[u][e].x, acc[4 * e]);
                acc[4 * e + 1] = fmaf(w, v4[u][e].y, acc[4 * e + 1]);
                acc[4 * e + 2] = fmaf(w, v4[u][e].z, acc[4 * e + 2]);
                acc[4 * e + 3] = fmaf(w, v4[u][e].w, acc[4 * e + 3]);
              }
            }
          }
          if (dfl) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
              reinterpret_cast<float4*>(dfl + cb * 32)[u] =
                  make_float4(acc[4 * u], acc[4 * u + 1], acc[4 * u + 2], acc[4 * u + 3]);
          } else if (dbf) {
#pragma unroll
            for (int e = 0; e < 32; e += 16) {
              uint32_t w8[8];
#pragma unroll
              for (int k2 = 0; k2 < 8; ++k2) w8[k2] = pack_bf16x2(acc[e + 2 * k2], acc[e + 2 * k2 + 1]);
              st_global_v8(dbf + cb * 32 + e, w8);
            }
          }
        }
        continue;
      }
      // the dense row's base-2 log-sum-exp, kept by the training forward
      if (p.lse_dense && row_valid && J.kind == JOB_DENSE_ROWS)
        p.lse_dense[((long long)J.b * p.H + h) * p.n_sel + gli] = (l_run > 0.f) ? m_run + __log2f(l_run) : -INFINITY;
      }  // !WIN
      const uint64_t inv2 = f2_pack(inv_l, inv_l);
      __nv_bfloat16* dst_bf = (store && mode_out == 0)
                                  ? p.out + (((long long)J.b * p.out_rows + out_row) * p.H + h) * HD
                                  : nullptr;
      float* dst_f = (store && mode_out != 0)
                         ? (mode_out == 1 ? p.dense_buf : p.sparse_buf) +
                               (((long long)J.b * p.n_anchor + gli) * p.H + h) * HD
                         : nullptr;
      // this tile's staging half is free once its last store has read it (the
      // leader waits for that store only now, so it never holds up the warps)
      const uint32_t half = base_u32 + G::STG_OFF + q * G::STG_HALF;
      if (use_stg || fuse) {
        if (quarter == 0 && lane == 0 && st_pending) {
          bulk_wait_read_all();
          mbar_arrive(BAR(stg_free[0]) + 8 * q);
          st_pending = false;
        }
        if (st_rounds > 0 &&
            !mbar_wait_warp(BAR(stg_free[0]) + 8 * q, (st_rounds - 1) & 1, wc, KERR_TIMEOUT_SOFTMAX))
          break;
      }
      // the anchor's bf16 delta row: written by the delta kernel (dlt) or,
      // fused, formed here by the warp that holds the anchor row
      const uint4* dsrc = reinterpret_cast<const uint4*>(dlt);
      if (pair) {
        if (q == 0) {
          // the slot is free once tile B has read the previous job's rows
          if (f_reads_prev > 0 &&
              !mbar_wait_warp(BAR(delta_free), (f_reads_prev - 1) & 1, wc, KERR_TIMEOUT_SOFTMAX))
            break;
          // lane 0's row is the anchor (position J.start).  Its raw O row goes
          // through the first 512 bytes of this warp's own staging rows; each
          // lane scales its 4 columns by the anchor's 1/l and forms dense - sparse
          float4* tmp = reinterpret_cast<float4*>(base + G::STG_OFF + quarter * 32 * 128);  // tile A's half
          if (lane == 0) {
#pragma unroll
            for (int c4 = 0; c4 < HD / 4; ++c4) tmp[c4] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
            reinterpret_cast<float*>(tmp)[HD] = inv_l;
          }
          __syncwarp();
          if (lane < HD / 4) {
            const float inv_l0 = reinterpret_cast<const float*>(tmp)[HD];
            const float4 ot = tmp[lane];
            const float4 d = make_float4(dn_first.x - ot.x * inv_l0, dn_first.y - ot.y * inv_l0,
                                         dn_first.z - ot.z * inv_l0, dn_first.w - ot.w * inv_l0);
            ctrl->dslot[quarter][2 * lane] = pack_bf16x2(d.x, d.y);
            ctrl->dslot[quarter][2 * lane + 1] = pack_bf16x2(d.z, d.w);
            if (p.anchor_delta_f32) reinterpret_cast<float4*>(p.anchor_delta_f32 + anchor_row * HD)[lane] = d;
          }
          __syncwarp();  // the slot is complete and the staging rows may be overwritten
          if (lane == 0) mbar_arrive(BAR(delta_ready));
        } else if (!mbar_wait_warp(BAR(delta_ready), f_writes_prev & 1, wc, KERR_TIMEOUT_SOFTMAX)) {
          break;
        }
        dsrc = reinterpret_cast<const uint4*>(&ctrl->dslot[quarter][0]);
      } else if (fuse) {
        // each anchor row of this warp: its raw O row and 1/l go through this
        // warp's own staging rows; each lane forms 4 columns of
        // dense - O / l (the sparse row exactly as the rows launch would store
        // it) and writes them to the anchor's delta slot
        float4* tmp = reinterpret_cast<float4*>(base + G::STG_OFF + q * G::STG_HALF + quarter * 32 * 128);
        uint32_t mask = anchor_mask;
        bool first = true;
        while (mask) {
          const int al = __ffs(mask) - 1;
          mask &= mask - 1;
          if (lane == al) {
#pragma unroll
            for (int c4 = 0; c4 < HD / 4; ++c4) tmp[c4] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
            reinterpret_cast<float*>(tmp)[HD] = inv_l;
          }
          __syncwarp();
          const long long arow = __shfl_sync(0xffffffffu, anchor_row, al);
          if (lane < HD / 4) {
            const float inv_l0 = reinterpret_cast<const float*>(tmp)[HD];
            const float4 ot = tmp[lane];
            const float4 dn = first ? dn_first : __ldcg(reinterpret_cast<const float4*>(p.dense_buf + arow * HD) + lane);
            const float4 d = make_float4(dn.x - ot.x * inv_l0, dn.y - ot.y * inv_l0, dn.z - ot.z * inv_l0,
                                         dn.w - ot.w * inv_l0);
            reinterpret_cast<uint2*>(p.delta_buf + arow * HD)[lane] = make_uint2(pack_bf16x2(d.x, d.y), pack_bf16x2(d.z, d.w));
            if (p.anchor_delta_f32) reinterpret_cast<float4*>(p.anchor_delta_f32 + arow * HD)[lane] = d;
          }
          __syncwarp();  // the staging rows may be reused
          first = false;
        }
        if (p.delta_cross) {
          if (anchor_mask) {
            // publish: this warp's delta rows are visible to the CTA
            __threadfence_block();
            __syncwarp();
            if (lane == 0) atomicAdd(&ctrl->delta_count, 1);
          } else {
            // the four warps of this period's forming tile have published
            if (!__all_sync(0xffffffffu, smem_wait_geq(&ctrl->delta_count, 4 * periods, wc, KERR_TIMEOUT_SOFTMAX)))
              break;
            __threadfence_block();
          }
        }
        dsrc = reinterpret_cast<const uint4*>(p.delta_buf + anchor_row * HD);
        // rows formed by this warp just now: into L1 ahead of the stores (the
        // rows are written and read by this SM only, in this launch)
        if (anchor_mask) {
#pragma unroll
          for (int c = 0; c < HD * 2 / 128; ++c)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const char*>(dsrc) + c * 128));
        }
      }
      auto dload = [&](int i) -> uint4 { return dsrc ? dsrc[i] : make_uint4(0, 0, 0, 0); };
      if (use_stg) {
        // row r of the tile (head r / R, position r % R: the order of the
        // (64, R, G, 1) box) as a 128-byte-swizzled 128-byte row of this tile's
        // staging half, 64 columns per round; o / l + delta on packed fp32 pairs
        bool ok = true;
#pragma unroll
        for (int rg = 0; rg < G::REGIONS; ++rg) {
          if (rg > 0 &&
              !mbar_wait_warp(BAR(stg_free[0]) + 8 * q, (st_rounds - 1) & 1, wc, KERR_TIMEOUT_SOFTMAX)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int cw = 0; cw < 8; ++cw) {
            const int c16 = rg * 8 + cw;
            const uint4 dv = dload(c16);
            const uint32_t dw4[4] = {dv.x, dv.y, dv.z, dv.w};
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int col = c16 * 8 + 2 * k;
              const uint64_t d2 = f2_pack(__uint_as_float(dw4[k] << 16), __uint_as_float(dw4[k] & 0xffff0000u));
              float a, b;
              f2_unpack(f2_fma(f2_pack(o[col], o[col + 1]), inv2, d2), a, b);
              w[k] = pack_bf16x2(a, b);
            }
            st_shared_v4(half + r * 128 + ((cw ^ (r & 7)) << 4), w[0], w[1], w[2], w[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(BAR(stg_full[0]) + 8 * q);
          if (quarter == 0 && lane == 0) {
            // leader: once all four warps wrote their rows, store the round; the
            // half is released when the store has read it (for the tile's last
            // round, at this tile's next use)
            ok = mbar_wait(BAR(stg_full[0]) + 8 * q, st_rounds & 1, wc, KERR_TIMEOUT_SOFTMAX);
            if (ok) {
              tma_store_4d(&p.tm_out, half, rg * 64, J.start + q * p.R, J.g * p.G, J.b);
              bulk_commit_group();
              if (rg + 1 < G::REGIONS) {
                bulk_wait_read_all();
                mbar_arrive(BAR(stg_free[0]) + 8 * q);
              } else {
                st_pending = true;
              }
            }
          }
          if (!__all_sync(0xffffffffu, ok)) break;
          ++st_rounds;
        }
        if (!ok) break;
      } else if (dst_bf) {
        // o / l + delta on packed fp32 pairs (one fma.rn.f32x2 per pair); the
        // delta row is shared by the warp's rows in the common case (L1 hits)
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t ww[16];
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            const uint4 w = dload(c * 4 + v4);
            ww[4 * v4] = w.x; ww[4 * v4 + 1] = w.y; ww[4 * v4 + 2] = w.z; ww[4 * v4 + 3] = w.w;
          }
#pragma unroll
          for (int e = 0; e < 32; e += 16) {
            uint32_t w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int kk = e / 2 + k;
              const uint64_t d2 = f2_pack(__uint_as_float(ww[kk] << 16), __uint_as_float(ww[kk] & 0xffff0000u));
              float a, b;
              f2_unpack(f2_fma(f2_pack(o[c * 32 + 2 * kk], o[c * 32 + 2 * kk + 1]), inv2, d2), a, b);
              w[k] = pack_bf16x2(a, b);
            }
            st_global_v8(dst_bf + c * 32 + e, w);
          }
        }
      } else if (dst_f) {
#pragma unroll
        for (int e = 0; e < HD; e += 4)
          *reinterpret_cast<float4*>(dst_f + e) =
              make_float4(o[e] * inv_l, o[e + 1] * inv_l, o[e + 2] * inv_l, o[e + 3] * inv_l);
      }
      if (pair && q == 1) {
        __syncwarp();  // every lane has read the slot
        if (lane == 0) mbar_arrive(BAR(delta_free));
      }
    }
  }
#undef BAR
  // bulk (TMA) stores of this thread complete before the CTA exits
  if (warp >= 4 && (warp & 3) == 0 && lane == 0) bulk_wait_all();
  // a windowed CTA never completes before the grid it depends on (also when
  // it read none of that grid's output)
  if (WIN && threadIdx.x == 0) grid_dependency_wait();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Geo<HD>::TMEM_COLS);
  }
}

template <int HD, int LK, int FM>
static cudaError_t launch_prefill_hd(const PrefillParams& p, int grid, bool dependent, cudaStream_t stream) {
  const int smem = Geo<HD>::SMEM_BYTES;
  cudaError_t e = cudaFuncSetAttribute(prefill_kernel<HD, LK, FM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, prefill_kernel<HD, LK, FM>, p);
}

cudaError_t launch_prefill(const PrefillParams& p, int head_dim, int grid, bool dependent, cudaStream_t stream) {
  const int fm = !p.fuse_delta ? FUSE_NONE : (p.delta_pair ? FUSE_PAIR : FUSE_GENERAL);
  if (p.launch != LAUNCH_WINDOW)
    return head_dim == 128 ? launch_prefill_hd<128, LAUNCH_ROWS, FUSE_NONE>(p, grid, false, stream)
                           : launch_prefill_hd<64, LAUNCH_ROWS, FUSE_NONE>(p, grid, false, stream);
  if (head_dim == 128) {
    if (fm == FUSE_PAIR) return launch_prefill_hd<128, LAUNCH_WINDOW, FUSE_PAIR>(p, grid, dependent, stream);
    if (fm == FUSE_GENERAL) return launch_prefill_hd<128, LAUNCH_WINDOW, FUSE_GENERAL>(p, grid, dependent, stream);
    return launch_prefill_hd<128, LAUNCH_WINDOW, FUSE_NONE>(p, grid, dependent, stream);
  }
  if (fm == FUSE_PAIR) return launch_prefill_hd<64, LAUNCH_WINDOW, FUSE_PAIR>(p, grid, dependent, stream);
  if (fm == FUSE_GENERAL) return launch_prefill_hd<64, LAUNCH_WINDOW, FUSE_GENERAL>(p, grid, dependent, stream);
  return launch_prefill_hd<64, LAUNCH_WINDOW, FUSE_NONE>(p, grid, dependent, stream);
}

}  // namespace dta
