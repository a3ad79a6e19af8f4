// Training backward of the delta-attention layer on sm_100a: the gradient of
// delta_attention/train/flex_delta.py:95-196 (delta_forward_train) with
// respect to q, k and v, for uniform anchors.
//
// Forward (per (batch, head)): sparse = A_W(q, k, v) over the block-anchored
// sink + window mask (every row below s_p), dense = A_D(q[sel], k, v) over
// the causal mask for the rows sel = anchors (0, gamma, ... < s_p) + tail
// (s_p .. s-1), delta = dense[anchor] - sparse[anchor],
// out[r] = sparse[r] + delta[r / gamma] (r < s_p), out[s_p + t] = dense[tail t].
// Backward with G = dL/dout:
//   g_delta[a] = c * sum_{j < gamma} G[a gamma + j]   (c = delta_grad_scale; 0 = detached)
//   dL/dsparse[r] = G[r] - (r = a gamma ? g_delta[a] : 0)   (rows < s_p)
//   dL/ddense[a] = g_delta[a];  dL/ddense[tail t] = G[s_p + t]
// and each attention's own backward with its saved base-2 log-sum-exp:
//   P = exp2(S * scale * log2(e) - lse),  D_r = sum_d dO[r] O[r],
//   dS = P (dP - D),  dP = dO V^T,  dV += P^T dO,  dK += scale dS^T Q,  dQ += scale dS K.
// O of the sparse pass is out - delta (rows < s_p), of the dense pass `out` at
// the dense rows, so the forward keeps only out, delta and the two lse arrays.
//
// Kernels (one stream, in order):
//   backward_prep    : g_delta, both passes' dO (bf16, head-major [b, H, rows, d]),
//                      D, and q of the dense rows in list order (so every tile
//                      load is one TMA box)
//   backward_plan    : per key tile, the first job of the key-major launch
//   bwd_kernel<QM>   : query-major, dense rows: a job is one list tile over
//                      its key tiles; dQ accumulates in TMEM (anchor rows to an
//                      fp32 buffer, tail rows to grad_q)
//   bwd_kernel<KM>   : key-major, queued as a programmatic dependent launch of
//                      the one before: a job is one key tile (128 keys of one
//                      KV group) and a chunk of the query tiles that attend
//                      it; dK, dV accumulate in TMEM and leave with fp32
//                      vector atomics (a key tile's chunks may run on several SMs)
//   bwd_kernel<QM>   : query-major, windowed rows (adds the dense rows' dQ of
//                      each anchor row)
//   backward_finalize: dK (times scale), dV to bf16
// Per (query tile, key tile) both tcgen05 kernels run S and dP as two
// SS-form 128 x 128 x d products and form P and dS in registers (two compute
// warpgroups, 64 columns each, packed fp32 pairs).  Key-major: P^T and then
// dS^T go back over S^T / dP^T in TMEM as bf16, in two phases with their own
// barriers, and feed TS-form products (A from TMEM, B an MN-major view of the
// shared-memory tile that S^T and dP^T read K-major); the issue order dV,
// next S^T, dK, next dP^T overlaps each phase with tensor work.  Query-major:
// dS goes to one of two spare TMEM buffers, and the next key tile's S and dP
// are issued as soon as this tile's S, respectively dP, is in registers.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cmath>

#include "dta_backward.h"
#include "dta_ptx.cuh"

namespace dta {

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
// One CTA per (anchor block or tail chunk, batch); thread u of a pass covers 8
// columns (head u / (d/8), columns 8 (u % (d/8)) ..).  A head's d/8 threads are
// consecutive lanes of one warp, so row sums reduce with shuffles.
constexpr int PREP_THREADS = 256;
constexpr int PREP_TAIL_ROWS = 16;

__device__ __forceinline__ void ld_bf16x8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void st_bf16x8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
// values as the tensor cores will see them (bf16-rounded)
__device__ __forceinline__ void round_bf16x8(float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const uint32_t w = pack_bf16x2(f[i], f[i + 1]);
    f[i] = __uint_as_float(w << 16);
    f[i + 1] = __uint_as_float(w & 0xffff0000u);
  }
}
// sum over the `n` lanes (a power of two, aligned) that hold one head's row
__device__ __forceinline__ float head_sum(float x, int n) {
  for (int o = n >> 1; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__global__ void __launch_bounds__(PREP_THREADS) backward_prep_kernel(
    const __nv_bfloat16* __restrict__ q, long long q_sb, long long q_sh, long long q_ss,
    const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ gout,
    const float* __restrict__ anchor_delta, __nv_bfloat16* __restrict__ g_sp, __nv_bfloat16* __restrict__ g_dn,
    __nv_bfloat16* __restrict__ q_sel, float* __restrict__ d_sp, float* __restrict__ d_dn, int H, int S, int d,
    int s_p, int n_anchor, int n_sel, int gamma, float gscale) {
  const int b = blockIdx.y;
  const int units = H * d / 8, per_head = d / 8;
  const long long row_el = (long long)H * d;  // elements per row of out / gout / g_*
  const int n_tail_blocks = (n_sel - n_anchor + PREP_TAIL_ROWS - 1) / PREP_TAIL_ROWS;
  // every lane of a warp runs the same number of passes (whole warps per head)
  for (int u0 = 0; u0 < units; u0 += PREP_THREADS) {
    const int u = u0 + (int)threadIdx.x;
    const bool act = u < units;
    const int h = act ? u / per_head : 0, c = act ? (u % per_head) * 8 : 0;
    if ((int)blockIdx.x < n_anchor) {
      const int a = blockIdx.x, r0 = a * gamma;
      // delta's gradient: the block's output gradients, summed
      float gd[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (act && gscale != 0.f) {
        for (int j = 0; j < gamma; ++j) {
          float f[8];
          ld_bf16x8(gout + ((long long)b * S + r0 + j) * row_el + h * d + c, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) gd[e] += f[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) gd[e] *= gscale;
      }
      round_bf16x8(gd);
      // dense pass, anchor row: dO = g_delta, O = out[anchor] (= dense[a])
      float o[8];
      if (act) {
        ld_bf16x8(out + ((long long)b * S + r0) * row_el + h * d + c, o);
        st_bf16x8(g_dn + (((long long)b * H + h) * n_sel + a) * d + c, gd);
        float qv[8];
        ld_bf16x8(q + b * q_sb + h * q_sh + r0 * q_ss + c, qv);
        st_bf16x8(q_sel + (((long long)b * H + h) * n_sel + a) * d + c, qv);
      }
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) dot += act ? gd[e] * o[e] : 0.f;
      dot = head_sum(dot, per_head);
      if (act && c == 0) d_dn[((long long)b * H + h) * n_sel + a] = dot;
      // sparse pass, rows of the block: dO = G - [anchor] g_delta, O = out - delta
      float dl[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (act) {
        const float4* dp = reinterpret_cast<const float4*>(anchor_delta + (((long long)b * n_anchor + a) * H + h) * d + c);
        const float4 x = dp[0], y = dp[1];
        dl[0] = x.x; dl[1] = x.y; dl[2] = x.z; dl[3] = x.w; dl[4] = y.x; dl[5] = y.y; dl[6] = y.z; dl[7] = y.w;
      }
      for (int j = 0; j < gamma; ++j) {
        const int r = r0 + j;
        float g[8], ov[8];
        float s = 0.f;
        if (act) {
          ld_bf16x8(gout + ((long long)b * S + r) * row_el + h * d + c, g);
          if (j == 0) {
#pragma unroll
            for (int e = 0; e < 8; ++e) g[e] -= gd[e];
          }
          round_bf16x8(g);
          st_bf16x8(g_sp + (((long long)b * H + h) * s_p + r) * d + c, g);
          ld_bf16x8(out + ((long long)b * S + r) * row_el + h * d + c, ov);
#pragma unroll
          for (int e = 0; e < 8; ++e) s += g[e] * (ov[e] - dl[e]);
        }
        s = head_sum(s, per_head);
        if (act && c == 0) d_sp[((long long)b * H + h) * S + r] = s;
      }
    } else {
      // dense tail rows: dO = G, O = out
      const int t0 = ((int)blockIdx.x - n_anchor) * PREP_TAIL_ROWS;
      if ((int)blockIdx.x - n_anchor >= n_tail_blocks) return;
      for (int t = t0; t < t0 + PREP_TAIL_ROWS && n_anchor + t < n_sel; ++t) {
        const int i = n_anchor + t, r = s_p + t;
        float g[8], ov[8];
        float s = 0.f;
        if (act) {
          ld_bf16x8(gout + ((long long)b * S + r) * row_el + h * d + c, g);
          st_bf16x8(g_dn + (((long long)b * H + h) * n_sel + i) * d + c, g);
          ld_bf16x8(out + ((long long)b * S + r) * row_el + h * d + c, ov);
#pragma unroll
          for (int e = 0; e < 8; ++e) s += g[e] * ov[e];
          float qv[8];
          ld_bf16x8(q + b * q_sb + h * q_sh + (long long)r * q_ss + c, qv);
          st_bf16x8(q_sel + (((long long)b * H + h) * n_sel + i) * d + c, qv);
        }
        s = head_sum(s, per_head);
        if (act && c == 0) d_dn[((long long)b * H + h) * n_sel + i] = s;
      }
    }
  }
}

cudaError_t launch_backward_prep(const __nv_bfloat16* q, long long q_sb, long long q_sh, long long q_ss,
                                 const __nv_bfloat16* out, const __nv_bfloat16* gout, const float* anchor_delta,
                                 __nv_bfloat16* g_sp, __nv_bfloat16* g_dn, __nv_bfloat16* q_sel, float* d_sp,
                                 float* d_dn, int B, int H, int S, int d, int s_p, int n_anchor, int n_sel, int gamma,
                                 float delta_grad_scale, cudaStream_t stream) {
  const int n_tail_blocks = (n_sel - n_anchor + PREP_TAIL_ROWS - 1) / PREP_TAIL_ROWS;
  const dim3 grid(n_anchor + n_tail_blocks, B);
  backward_prep_kernel<<<grid, PREP_THREADS, 0, stream>>>(q, q_sb, q_sh, q_ss, out, gout, anchor_delta, g_sp, g_dn,
                                                          q_sel, d_sp, d_dn, H, S, d, s_p, n_anchor, n_sel, gamma,
                                                          delta_grad_scale);
  return cudaGetLastError();
}

// chunk_base[kt] = first chunk of key tile kt in the key-major launch: each of
// the 1024 threads counts the chunks of a run of consecutive key tiles, then a
// block-wide exclusive scan (warp shuffles, then the 32 warp totals) places them
constexpr int PLAN_THREADS = 1024;

__global__ void __launch_bounds__(PLAN_THREADS) backward_plan_kernel(int* chunk_base, int n_ktiles, int S, int s_p,
                                                                     int n_anchor, int n_sel, int gamma, int window,
                                                                     int sink, int qblock, int R, int chunk_iters) {
  __shared__ int warp_tot[PLAN_THREADS / 32];
  const int per = (n_ktiles + PLAN_THREADS - 1) / PLAN_THREADS;
  const int t0 = threadIdx.x * per, t1 = min(t0 + per, n_ktiles);
  auto chunks = [&](int kt) {
    const KeyTileList L = bwd_key_tile_list(kt, S, s_p, n_anchor, n_sel, gamma, window, sink, qblock, R);
    return ((L.us1 - L.us0) + (L.ud1 - L.ud0) + chunk_iters - 1) / chunk_iters;
  };
  int mine = 0;
  for (int kt = t0; kt < t1; ++kt) mine += chunks(kt);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = mine;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tot[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_tot[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  int acc = (warp > 0 ? warp_tot[warp - 1] : 0) + incl - mine;  // exclusive prefix of this thread's run
  for (int kt = t0; kt < t1; ++kt) {
    chunk_base[kt] = acc;
    acc += chunks(kt);
  }
  if (threadIdx.x == PLAN_THREADS - 1) chunk_base[n_ktiles] = warp_tot[31];
}

cudaError_t launch_backward_plan(int* chunk_base, int n_ktiles, int S, int s_p, int n_anchor, int n_sel, int gamma,
                                 int window, int sink, int qblock, int R, int chunk_iters, cudaStream_t stream) {
  backward_plan_kernel<<<1, PLAN_THREADS, 0, stream>>>(chunk_base, n_ktiles, S, s_p, n_anchor, n_sel, gamma, window,
                                                       sink, qblock, R, chunk_iters);
  return cudaGetLastError();
}

__global__ void backward_finalize_kernel(const float4* __restrict__ dk_acc, const float4* __restrict__ dv_acc,
                                         uint2* __restrict__ dk, uint2* __restrict__ dv, long long n4, float scaling) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 a = dk_acc[i], b = dv_acc[i];
    dk[i] = make_uint2(pack_bf16x2(a.x * scaling, a.y * scaling), pack_bf16x2(a.z * scaling, a.w * scaling));
    dv[i] = make_uint2(pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
  }
}

cudaError_t launch_backward_finalize(const float* dk_acc, const float* dv_acc, __nv_bfloat16* dk, __nv_bfloat16* dv,
                                     long long n, float scaling, cudaStream_t stream) {
  const long long n4 = n / 4;
  long long blocks = (n4 + 255) / 256;
  if (blocks > 8192) blocks = 8192;
  if (blocks < 1) blocks = 1;
  backward_finalize_kernel<<<(int)blocks, 256, 0, stream>>>(reinterpret_cast<const float4*>(dk_acc),
                                                            reinterpret_cast<const float4*>(dv_acc),
                                                            reinterpret_cast<uint2*>(dk), reinterpret_cast<uint2*>(dv),
                                                            n4, scaling);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// the tcgen05 backward kernel (both launches)
// ---------------------------------------------------------------------------
// 384 threads, one CTA per SM:
//   warp 0      producer: fetches jobs, publishes each with its iteration
//               range, loads the job's two fixed tiles (A operands: q and dO
//               of the query tile, or k and v of the key tile) and streams the
//               other operand pair (k, v tiles / q, dO tiles with the query
//               rows' lse and D) through two stages
//   warp 1      TMEM owner and MMA issuer (one elected lane issues)
//   warps 2, 3  idle
//   warps 4..11 two compute warpgroups; warpgroup w owns columns [64 w, 64 w + 64)
//               of S and dP (TMEM lane = the thread's tile row)
// TMEM: T1 [0, 128) S or S^T (key-major: then bf16 P^T in place); T2 [128,
// 256) dP or dP^T (key-major: then bf16 dS^T in place); accumulators from
// column 256: dQ, or dV then dK; query-major: bf16 dS buffers at 384 and 448.
constexpr int BWD_THREADS = 384;
constexpr int BWD_CTRL = 1024;
enum BwdKind : int { BWD_QM = 0, BWD_KM = 1 };

template <int HD>
struct BGeo {
  static constexpr int REGIONS = HD / 64;
  static constexpr int REGION = 128 * 128;           // 128 rows x 128 bytes (64 bf16 columns)
  static constexpr int TILE = REGIONS * REGION;      // 128 rows x HD bf16
  static constexpr int STATS = 1024;                 // key-major stage: lse[128], D[128]
  static constexpr int STAGE = 2 * TILE + STATS;
  static constexpr int NST = 2;
  static constexpr int FIX_OFF = BWD_CTRL;
  static constexpr int STR_OFF = FIX_OFF + 2 * TILE;
  static constexpr int SMEM = STR_OFF + NST * STAGE + 1024;  // + alignment slack
  // query-major: separate rings, K for three iterations (read by S and by dQ),
  // V for two (read by dP only, released as soon as dP is done)
  static constexpr int KST = 3, VST = 2;
  static constexpr int K_OFF = FIX_OFF + 2 * TILE;
  static constexpr int V_OFF = K_OFF + KST * TILE;
  static constexpr int SMEM_QM = V_OFF + VST * TILE + 1024;
  static constexpr int T1 = 0, T2 = 128, ACC1 = 256, ACC2 = 256 + HD;
  static constexpr int DS = 384;  // query-major: two bf16 dS buffers of 64 columns
};
static_assert(BGeo<128>::SMEM <= 232448 && BGeo<128>::SMEM_QM <= 232448, "shared memory budget");
static_assert(BGeo<128>::STAGE % 1024 == 0 && BGeo<64>::STAGE % 1024 == 0, "tiles stay 1024-byte aligned");

struct BCtrl {
  uint64_t job_full[2], job_empty[2];
  uint64_t fix_full, fix_empty;
  uint64_t st_full[2], st_empty[2];
  uint64_t s_full, p_full, acc_full, acc_empty;
  uint64_t dp_full, ds_full;  // key-major: dP^T is in T2; dS^T has been written over it
  uint64_t k_full[3], k_empty[3], v_full[2], v_empty[2];  // query-major rings
  uint64_t s_free;      // query-major: S of the iteration is in registers (T1 free)
  uint64_t dp_free;     // query-major: dP of the iteration is in registers (T2 free)
  uint64_t ds_free[2];  // query-major: the dQ product has read dS buffer b
  uint64_t drain;
  // job record: [0] kind (1 job, -1 end), [1] b, [2] g, [3] tile, [4] i0,
  // [5] i1, [6] n0, [7] w0, [8] us0, [9] us1, [10] ud0
  int job[2][12];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(BCtrl) <= BWD_CTRL, "control block too large");

struct BJob {
  int kind, b, g, tile, i0, i1, n0, w0, us0, us1, ud0;
};

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// bits [lo, hi) of a 32-bit word (clamped)
__device__ __forceinline__ uint32_t bits_range(int lo, int hi) {
  const uint32_t a = lo <= 0 ? 0xffffffffu : (lo >= 32 ? 0u : (0xffffffffu << lo));
  const uint32_t b = hi <= 0 ? 0xffffffffu : (hi >= 32 ? 0u : (0xffffffffu << hi));
  return a & ~b;
}

__device__ __forceinline__ int blocklast(int t, int qblock) { return (t / qblock) * qblock + qblock - 1; }

// query-major job j of this launch's pass: the tile, its key-tile plan
__device__ BJob bwd_decode_qm(const BackwardParams& p, int j) {
  BJob J{};
  const int BG = p.B * p.Hkv;
  if (j >= p.n_jobs) {
    J.kind = -1;
    return J;
  }
  J.kind = 1;
  const int bg = j % BG;
  J.b = bg / p.Hkv;
  J.g = bg - J.b * p.Hkv;
  if (p.pass == BWD_DENSE) {
    J.tile = p.n_qtiles - 1 - j / BG;  // longest (the tail) first
    const int last = min((J.tile + 1) * p.R, p.n_sel) - 1;
    const int kl = bwd_list_pos(last, p.gamma, p.n_anchor, p.s_p) / BWD_BN;
    J.n0 = kl + 1;
    J.w0 = J.n0;
    J.i1 = kl + 1;
  } else {
    J.tile = j / BG;
    const int first = J.tile * p.R;
    const int last = min(first + p.R, p.s_p) - 1;
    const int kl = last / BWD_BN;
    const int lo = max(0, blocklast(first, p.qblock) - p.window + 1);
    const int nst = (p.sink + BWD_BN - 1) / BWD_BN;
    const int w0 = lo / BWD_BN;
    if (w0 <= nst) {
      J.n0 = kl + 1;
      J.w0 = J.n0;
      J.i1 = kl + 1;
    } else {
      J.n0 = min(nst, kl + 1);
      J.w0 = w0;
      J.i1 = J.n0 + (kl - w0 + 1);
    }
  }
  J.i0 = 0;
  return J;
}

// key-major job j: key tile, chunk of its query-tile list
__device__ BJob bwd_decode_km(const BackwardParams& p, int j) {
  BJob J{};
  if (j >= p.n_jobs) {
    J.kind = -1;
    return J;
  }
  J.kind = 1;
  const int bg = j / p.total_chunks, c = j - bg * p.total_chunks;
  J.b = bg / p.Hkv;
  J.g = bg - J.b * p.Hkv;
  int lo = 0, hi = p.n_ktiles - 1;  // largest kt with chunk_base[kt] <= c
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.chunk_base[mid] <= c) lo = mid;
    else hi = mid - 1;
  }
  J.tile = lo;
  const KeyTileList L = bwd_key_tile_list(lo, p.S, p.s_p, p.n_anchor, p.n_sel, p.gamma, p.window, p.sink, p.qblock, p.R);
  const int n = (L.us1 - L.us0) + (L.ud1 - L.ud0);
  J.i0 = (c - p.chunk_base[lo]) * p.chunk_iters;
  J.i1 = min(J.i0 + p.chunk_iters, n);
  J.us0 = L.us0;
  J.us1 = L.us1;
  J.ud0 = L.ud0;
  return J;
}

template <int HD, int KIND>
__global__ void __launch_bounds__(BWD_THREADS, 1) bwd_kernel(const __grid_constant__ BackwardParams p) {
  using G = BGeo<HD>;
  constexpr bool KM = (KIND == BWD_KM);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - raw_u32);
  BCtrl* ctrl = reinterpret_cast<BCtrl*>(base);
  const uint32_t ctrl_u32 = base_u32;
#define BBAR(field) (ctrl_u32 + (uint32_t)offsetof(BCtrl, field))
  const uint32_t fix_u32 = base_u32 + G::FIX_OFF;  // fixed tile 0 at +0, tile 1 at +TILE
  const uint32_t str_u32 = base_u32 + G::STR_OFF;  // stage s: tile 0, tile 1, stats
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &ctrl->abort_flag;
  const WaitCtx wc{abort_flag, p.error, p.wait_cycles};

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(BBAR(job_full[0]) + 8 * i, 1);
      mbar_init(BBAR(job_empty[0]) + 8 * i, 1 + 8);  // MMA warp lane 0 + 8 compute warps
      mbar_init(BBAR(st_full[0]) + 8 * i, 2);  // the copies' expect_tx arrival + the stats' arrival
      mbar_init(BBAR(st_empty[0]) + 8 * i, 1);
    }
    mbar_init(BBAR(fix_full), 1);
    mbar_init(BBAR(fix_empty), 1);
    mbar_init(BBAR(s_full), 1);
    mbar_init(BBAR(p_full), 8);
    mbar_init(BBAR(acc_full), 1);
    mbar_init(BBAR(acc_empty), 8);
    mbar_init(BBAR(dp_full), 1);
    mbar_init(BBAR(ds_full), 8);
    for (int i = 0; i < 3; ++i) {
      mbar_init(BBAR(k_full[0]) + 8 * i, 1);
      mbar_init(BBAR(k_empty[0]) + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(BBAR(v_full[0]) + 8 * i, 1);
      mbar_init(BBAR(v_empty[0]) + 8 * i, 1);
    }
    mbar_init(BBAR(s_free), 8);
    mbar_init(BBAR(dp_free), 8);
    mbar_init(BBAR(ds_free[0]), 1);
    mbar_init(BBAR(ds_free[0]) + 8, 1);
    mbar_init(BBAR(drain), 1);
    ctrl->abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_qsel);
    tma_prefetch_desc(&p.tm_gsp);
    tma_prefetch_desc(&p.tm_gdn);
  }
  // the dense-row dQ launch lets the key-major launch queued behind it start
  // its CTAs as this grid's CTAs finish (its longest job, the tail rows over
  // every key tile, would otherwise leave most SMs idle at the end)
  if (!KM && p.pass == BWD_DENSE && threadIdx.x == 0) grid_dependents_launch();
  __syncwarp();
  if (warp == 1) {
    tmem_alloc(BBAR(tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  constexpr uint32_t IDESC_SS = idesc_bf16_f32(128, 128, 0);
  constexpr uint32_t IDESC_TS = idesc_bf16_f32(128, HD, 1);
  const int r_shift = __ffs(p.R) - 1;  // R = 128 / G, a power of two

  if (warp == 0) {
    // ======================= producer =======================
    int n = 0;            // stream items issued (stage ring position)
    int nk = 0, nv = 0;   // query-major: K / V loads issued (for the drain on abort)
    int jobs = 0;         // jobs whose fixed tiles were loaded
    bool ok = true;
    for (int it = 0; ok; ++it) {
      const int slot = it & 1;
      BJob J;
      {
        int jj = 0;
        for (;;) {
          if (lane == 0) jj = atomicAdd(p.counter, 1);
          jj = __shfl_sync(0xffffffffu, jj, 0);
          J = KM ? bwd_decode_km(p, jj) : bwd_decode_qm(p, jj);
          if (J.kind < 0 || J.i1 > J.i0) break;  // (a job without iterations is skipped)
        }
      }
      if (!mbar_wait_warp(BBAR(job_empty[0]) + 8 * slot, ((it >> 1) & 1) ^ 1, wc, KERR_TIMEOUT_PRODUCER)) break;
      if (lane == 0) {
        int* dst = ctrl->job[slot];
        dst[0] = J.kind; dst[1] = J.b; dst[2] = J.g; dst[3] = J.tile; dst[4] = J.i0; dst[5] = J.i1;
        dst[6] = J.n0; dst[7] = J.w0; dst[8] = J.us0; dst[9] = J.us1; dst[10] = J.ud0;
        mbar_arrive(BBAR(job_full[0]) + 8 * slot);
      }
      if (J.kind < 0) break;
      // the job's fixed tiles (A operands)
      if (!mbar_wait_warp(BBAR(fix_empty), (jobs & 1) ^ 1, wc, KERR_TIMEOUT_PRODUCER)) break;
      ++jobs;
      if (lane == 0) {
        mbar_arrive_expect_tx(BBAR(fix_full), 2 * G::TILE);
        for (int rg = 0; rg < G::REGIONS; ++rg) {
          const uint32_t d0 = fix_u32 + rg * G::REGION, d1 = fix_u32 + G::TILE + rg * G::REGION;
          if constexpr (KM) {
            tma_load_4d(d0, &p.tm_k, BBAR(fix_full), rg * 64, J.tile * BWD_BN, J.g, J.b);
            tma_load_4d(d1, &p.tm_v, BBAR(fix_full), rg * 64, J.tile * BWD_BN, J.g, J.b);
          } else if (p.pass == BWD_DENSE) {
            tma_load_4d(d0, &p.tm_qsel, BBAR(fix_full), rg * 64, J.tile * p.R, J.g * p.G, J.b);
            tma_load_4d(d1, &p.tm_gdn, BBAR(fix_full), rg * 64, J.tile * p.R, J.g * p.G, J.b);
          } else {
            tma_load_4d(d0, &p.tm_q, BBAR(fix_full), rg * 64, J.tile * p.R, J.g * p.G, J.b);
            tma_load_4d(d1, &p.tm_gsp, BBAR(fix_full), rg * 64, J.tile * p.R, J.g * p.G, J.b);
          }
        }
      }
      if constexpr (!KM) {
        // query-major: K and V of every key tile through their rings
        for (int u = J.i0; u < J.i1; ++u, ++n) {
          const int kt = u < J.n0 ? u : J.w0 + (u - J.n0);
          const int ks = n % G::KST, vs = n % G::VST;
          if (!mbar_wait_warp(BBAR(k_empty[0]) + 8 * ks, ((n / G::KST) & 1) ^ 1, wc, KERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            const uint32_t kd = base_u32 + G::K_OFF + ks * G::TILE;
            mbar_arrive_expect_tx(BBAR(k_full[0]) + 8 * ks, G::TILE);
            for (int rg = 0; rg < G::REGIONS; ++rg)
              tma_load_4d(kd + rg * G::REGION, &p.tm_k, BBAR(k_full[0]) + 8 * ks, rg * 64, kt * BWD_BN, J.g, J.b);
          }
          nk = n + 1;
          if (!mbar_wait_warp(BBAR(v_empty[0]) + 8 * vs, ((n / G::VST) & 1) ^ 1, wc, KERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            const uint32_t vd = base_u32 + G::V_OFF + vs * G::TILE;
            mbar_arrive_expect_tx(BBAR(v_full[0]) + 8 * vs, G::TILE);
            for (int rg = 0; rg < G::REGIONS; ++rg)
              tma_load_4d(vd + rg * G::REGION, &p.tm_v, BBAR(v_full[0]) + 8 * vs, rg * 64, kt * BWD_BN, J.g, J.b);
          }
          nv = n + 1;
        }
      } else {
      // key-major: the streamed operand pair (q, dO tiles and their rows' lse, D)
      for (int u = J.i0; u < J.i1; ++u, ++n) {
        const int st = n & 1;
        // query rows of this iteration: their lse and D, loaded before the
        // wait for the ring slot so that their latency overlaps it (columns
        // the tile does not have: lse = +inf, D = 0)
        const int ns = J.us1 - J.us0;
        const bool dense = u >= ns;
        const int qt = dense ? J.ud0 + (u - ns) : J.us0 + u;
        float lse[4], dv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int m = lane + 32 * k;
          const int hh = m >> r_shift, rr = m & (p.R - 1);
          const int head = J.g * p.G + hh;
          const int row = qt * p.R + rr;
          lse[k] = INFINITY;
          dv[k] = 0.f;
          if (!dense && row < p.s_p) {
            const long long o = ((long long)J.b * p.H + head) * p.S + row;
            lse[k] = p.lse_sp[o];
            dv[k] = p.d_sp[o];
          } else if (dense && row < p.n_sel) {
            const long long o = ((long long)J.b * p.H + head) * p.n_sel + row;
            lse[k] = p.lse_dn[o];
            dv[k] = p.d_dn[o];
          }
        }
        if (!mbar_wait_warp(BBAR(st_empty[0]) + 8 * st, ((n >> 1) & 1) ^ 1, wc, KERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        const uint32_t s0 = str_u32 + st * G::STAGE, s1 = s0 + G::TILE;
        float* stats = reinterpret_cast<float*>(base + G::STR_OFF + st * G::STAGE + 2 * G::TILE);
        // the tiles' copies, then the stats, which add the barrier's second arrival
        if (lane == 0) {
          mbar_arrive_expect_tx(BBAR(st_full[0]) + 8 * st, 2 * G::TILE);
          for (int rg = 0; rg < G::REGIONS; ++rg) {
            if (dense) {
              tma_load_4d(s0 + rg * G::REGION, &p.tm_qsel, BBAR(st_full[0]) + 8 * st, rg * 64, qt * p.R, J.g * p.G, J.b);
              tma_load_4d(s1 + rg * G::REGION, &p.tm_gdn, BBAR(st_full[0]) + 8 * st, rg * 64, qt * p.R, J.g * p.G, J.b);
            } else {
              tma_load_4d(s0 + rg * G::REGION, &p.tm_q, BBAR(st_full[0]) + 8 * st, rg * 64, qt * p.R, J.g * p.G, J.b);
              tma_load_4d(s1 + rg * G::REGION, &p.tm_gsp, BBAR(st_full[0]) + 8 * st, rg * 64, qt * p.R, J.g * p.G, J.b);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          stats[lane + 32 * k] = -lse[k];  // negated: the compute warps form s * scale - lse with one packed fma
          stats[128 + lane + 32 * k] = dv[k];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(BBAR(st_full[0]) + 8 * st);
      }
      }
    }
    // on abort, loads in flight land before the CTA can exit: the last stage
    // of each ring position and the last fixed load (each waited for its slot)
    if (*abort_flag && lane == 0) {
      auto drain = [](uint32_t bar, uint32_t parity) {
        const long long t0 = clock64();
        while (!mbar_try_wait(bar, parity))
          if (clock64() - t0 > kWaitTimeoutCycles) break;
      };
      if constexpr (KM) {
        for (int m = max(0, n - G::NST); m < n; ++m) drain(BBAR(st_full[0]) + 8 * (m & 1), (uint32_t)((m >> 1) & 1));
      } else {
        for (int m = max(0, nk - G::KST); m < nk; ++m)
          drain(BBAR(k_full[0]) + 8 * (m % G::KST), (uint32_t)((m / G::KST) & 1));
        for (int m = max(0, nv - G::VST); m < nv; ++m)
          drain(BBAR(v_full[0]) + 8 * (m % G::VST), (uint32_t)((m / G::VST) & 1));
      }
      if (jobs > 0) drain(BBAR(fix_full), (uint32_t)((jobs - 1) & 1));
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    const uint64_t fdesc0 = smem_desc_sw128(fix_u32, 16, 1024);           // fixed tile 0, K-major
    const uint64_t fdesc1 = smem_desc_sw128(fix_u32 + G::TILE, 16, 1024);
    int n = 0, jobs = 0;
    bool aborted = false;
    for (int it = 0; !aborted; ++it) {
      const int slot = it & 1;
      if (!mbar_poll(BBAR(job_full[0]) + 8 * slot, (it >> 1) & 1, wc, KERR_TIMEOUT_MMA)) break;
      int i0, i1;
      bool end;
      {
        const volatile int* src = ctrl->job[slot];
        end = src[0] < 0;
        i0 = src[4];
        i1 = src[5];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BBAR(job_empty[0]) + 8 * slot);
      if (end) break;
      if (!mbar_poll(BBAR(fix_full), jobs & 1, wc, KERR_TIMEOUT_MMA)) break;
      if constexpr (!KM) {
        // Query-major, pipelined: S of iteration m + 1 is issued as soon as
        // the compute warpgroups hold iteration m's S in registers (s_free)
        // and dP(m + 1) once they hold dP(m) (dp_free), both before dQ(m);
        // dS(m) lives in its own TMEM buffer (DS + 64 (m & 1)), so dQ(m) and
        // S(m + 1) do not share columns.
        auto issue_ss = [&](int m) -> bool {
          const int ks = m % G::KST, vs = m % G::VST;
          if (!mbar_poll(BBAR(k_full[0]) + 8 * ks, (m / G::KST) & 1, wc, KERR_TIMEOUT_MMA)) return false;
          if (!mbar_poll(BBAR(v_full[0]) + 8 * vs, (m / G::VST) & 1, wc, KERR_TIMEOUT_MMA)) return false;
          if (m > 0 && !mbar_poll(BBAR(s_free), (m - 1) & 1, wc, KERR_TIMEOUT_MMA)) return false;
          tc_fence_after();
          const uint32_t s0 = base_u32 + G::K_OFF + ks * G::TILE, s1 = base_u32 + G::V_OFF + vs * G::TILE;
          const uint64_t sdesc0 = smem_desc_sw128(s0, 16, 1024), sdesc1 = smem_desc_sw128(s1, 16, 1024);
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint32_t off = ((kk >> 2) * G::REGION + (kk & 3) * 32) >> 4;
              umma_ss(tmem + G::T1, fdesc0 + off, sdesc0 + off, IDESC_SS, kk > 0 ? 1u : 0u);
            }
            umma_commit(BBAR(s_full));
          }
          __syncwarp();
          if (m > 0 && !mbar_poll(BBAR(dp_free), (m - 1) & 1, wc, KERR_TIMEOUT_MMA)) return false;
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint32_t off = ((kk >> 2) * G::REGION + (kk & 3) * 32) >> 4;
              umma_ss(tmem + G::T2, fdesc1 + off, sdesc1 + off, IDESC_SS, kk > 0 ? 1u : 0u);
            }
            umma_commit(BBAR(dp_full));
            umma_commit(BBAR(v_empty[0]) + 8 * vs);  // V is read by dP only
          }
          __syncwarp();
          return true;
        };
        auto issue_ts = [&](int m, bool first, bool last) -> bool {
          const int ks = m % G::KST;
          if (!mbar_poll(BBAR(p_full), m & 1, wc, KERR_TIMEOUT_MMA)) return false;
          if (first && jobs > 0 && !mbar_poll(BBAR(acc_empty), (jobs - 1) & 1, wc, KERR_TIMEOUT_MMA)) return false;
          tc_fence_after();
          const uint64_t mdesc0 = smem_desc_sw128(base_u32 + G::K_OFF + ks * G::TILE, G::REGION, 1024);
          const uint32_t ds = tmem + G::DS + (uint32_t)(m & 1) * 64;
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_ts(tmem + G::ACC1, ds + kk * 8, mdesc0 + ((kk * 2048) >> 4), IDESC_TS, (!first || kk > 0) ? 1u : 0u);
            umma_commit(BBAR(k_empty[0]) + 8 * ks);
            umma_commit(BBAR(ds_free[0]) + 8 * (m & 1));
            if (last) umma_commit(BBAR(acc_full));
          }
          __syncwarp();
          return true;
        };
        const int T = i1 - i0;
        if (!issue_ss(n)) break;
        for (int k = 0; k < T; ++k) {
          if (k + 1 < T) {
            if (!issue_ss(n + k + 1)) {
              aborted = true;
              break;
            }
          } else {
            // the job's fixed tiles are read by its S / dP products only
            if (elect_one()) umma_commit(BBAR(fix_empty));
            __syncwarp();
          }
          if (!issue_ts(n + k, k == 0, k == T - 1)) {
            aborted = true;
            break;
          }
        }
        if (aborted) break;
        n += T;
        ++jobs;
      } else {
      // Key-major: dV(m) is issued as soon as P^T(m) has been written over
      // S^T(m) in T1, S^T(m + 1) right behind it (the tensor pipe runs in
      // issue order, so it overwrites T1 only after dV(m) has read it), dK(m)
      // once dS^T(m) is over dP^T(m) in T2, then dP^T(m + 1) into the T2
      // dK(m) has read.  The compute warpgroups thus form dS^T(m) while the
      // pipe runs dV(m) and S^T(m + 1), and P^T(m + 1) while it runs dK(m) and
      // dP^T(m + 1).  (The stage of m + 1 must be in place early: its rows'
      // statistics are loaded before the producer waits for the ring slot.)
      auto issue_s = [&](int m) -> bool {  // S^T(m) = F0 . Q(m)^T into T1
        const int st = m & 1;
        if (!mbar_poll(BBAR(st_full[0]) + 8 * st, (m >> 1) & 1, wc, KERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint64_t sdesc0 = smem_desc_sw128(str_u32 + st * G::STAGE, 16, 1024);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * G::REGION + (kk & 3) * 32) >> 4;
            umma_ss(tmem + G::T1, fdesc0 + off, sdesc0 + off, IDESC_SS, kk > 0 ? 1u : 0u);
          }
          umma_commit(BBAR(s_full));
        }
        __syncwarp();
        return true;
      };
      auto issue_dp = [&](int m, bool last_of_job) {  // dP^T(m) = F1 . dO(m)^T into T2 (stage already full)
        const uint64_t sdesc1 = smem_desc_sw128(str_u32 + (m & 1) * G::STAGE + G::TILE, 16, 1024);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * G::REGION + (kk & 3) * 32) >> 4;
            umma_ss(tmem + G::T2, fdesc1 + off, sdesc1 + off, IDESC_SS, kk > 0 ? 1u : 0u);
          }
          umma_commit(BBAR(dp_full));
          // the job's fixed tiles are read by its S^T / dP^T products only
          if (last_of_job) umma_commit(BBAR(fix_empty));
        }
        __syncwarp();
      };
      const int T = i1 - i0;
      if (!issue_s(n)) break;
      issue_dp(n, T == 1);
      for (int k = 0; k < T; ++k) {
        const int m = n + k, st = m & 1;
        const uint32_t s0 = str_u32 + st * G::STAGE, s1 = s0 + G::TILE;
        if (!mbar_poll(BBAR(p_full), m & 1, wc, KERR_TIMEOUT_MMA)) {
          aborted = true;
          break;
        }
        if (k == 0 && jobs > 0 && !mbar_poll(BBAR(acc_empty), (jobs - 1) & 1, wc, KERR_TIMEOUT_MMA)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        // accumulators += (bf16 from T1 / T2) . stage tile (MN-major view)
        const uint64_t mdesc0 = smem_desc_sw128(s0, G::REGION, 1024), mdesc1 = smem_desc_sw128(s1, G::REGION, 1024);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t acol = kk < 4 ? kk * 8 : 64 + (kk - 4) * 8;
            umma_ts(tmem + G::ACC1, tmem + G::T1 + acol, mdesc1 + ((kk * 2048) >> 4), IDESC_TS,
                    (k > 0 || kk > 0) ? 1u : 0u);  // dV += P^T dO
          }
        }
        __syncwarp();
        if (k + 1 < T && !issue_s(m + 1)) {
          aborted = true;
          break;
        }
        if (!mbar_poll(BBAR(ds_full), m & 1, wc, KERR_TIMEOUT_MMA)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t acol = kk < 4 ? kk * 8 : 64 + (kk - 4) * 8;
            umma_ts(tmem + G::ACC2, tmem + G::T2 + acol, mdesc0 + ((kk * 2048) >> 4), IDESC_TS,
                    (k > 0 || kk > 0) ? 1u : 0u);  // dK += dS^T Q
          }
          umma_commit(BBAR(st_empty[0]) + 8 * st);
          if (k == T - 1) umma_commit(BBAR(acc_full));
        }
        __syncwarp();
        if (k + 1 < T) issue_dp(m + 1, k + 1 == T - 1);
      }
      if (aborted) break;
      n += T;
      ++jobs;
      }
    }
    __syncwarp();
    if (elect_one()) umma_commit(BBAR(drain));
    __syncwarp();
    const long long t0 = clock64();
    while (!mbar_try_wait(BBAR(drain), 0)) {
      if (clock64() - t0 > kWaitTimeoutCycles) {
        atomicCAS(p.error, 0, KERR_TIMEOUT_DRAIN);
        break;
      }
    }
  } else if (warp >= 4) {
    // ======================= compute =======================
    const int wg = (warp - 4) >> 2;   // column half of S / dP
    const int quarter = warp & 3;     // TMEM lane quarter
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    int n = 0, jobs = 0;
    for (int it = 0;; ++it) {
      const int slot = it & 1;
      if (!mbar_wait_warp(BBAR(job_full[0]) + 8 * slot, (it >> 1) & 1, wc, KERR_TIMEOUT_SOFTMAX)) break;
      BJob J;
      {
        const volatile int* src = ctrl->job[slot];
        J.kind = src[0]; J.b = src[1]; J.g = src[2]; J.tile = src[3]; J.i0 = src[4]; J.i1 = src[5];
        J.n0 = src[6]; J.w0 = src[7]; J.us0 = src[8]; J.us1 = src[9]; J.ud0 = src[10];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(BBAR(job_empty[0]) + 8 * slot);
      if (J.kind < 0) break;
      // this thread's row of the tile
      const int hh = r >> r_shift, rr = r & (p.R - 1);
      // query-major: the query row (position, lse, D, window start)
      int qpos = 0, qlo = 0;
      bool qvalid = false;
      float qlse = INFINITY, qd = 0.f;
      // key-major: the key, its sparse query range [klo, khi) and first dense list row
      int key = 0, klo = 0, khi = 0, kfirst = 0;
      if constexpr (KM) {
        key = J.tile * BWD_BN + r;
        if (key < p.S) {
          klo = key;
          khi = p.s_p;
          if (key >= p.sink) khi = (int)min((long long)p.s_p, bwd_window_end(key, p.window, p.qblock));
          kfirst = bwd_first_list_index(key, p.gamma, p.n_anchor, p.s_p);
        } else {
          klo = khi = 0;
          kfirst = p.n_sel;
        }
      } else {
        const int head = J.g * p.G + hh;
        if (p.pass == BWD_DENSE) {
          const int i = J.tile * p.R + rr;
          qvalid = i < p.n_sel;
          qpos = bwd_list_pos(min(i, p.n_sel - 1), p.gamma, p.n_anchor, p.s_p);
          if (qvalid) {
            const long long o = ((long long)J.b * p.H + head) * p.n_sel + i;
            qlse = p.lse_dn[o];
            qd = p.d_dn[o];
          }
        } else {
          qpos = J.tile * p.R + rr;
          qvalid = qpos < p.s_p;
          qlo = blocklast(qpos, p.qblock) - p.window + 1;
          if (qvalid) {
            const long long o = ((long long)J.b * p.H + head) * p.S + qpos;
            qlse = p.lse_sp[o];
            qd = p.d_sp[o];
          }
        }
      }
      bool aborted = false;
      if constexpr (!KM) {
        // query-major: take S of the iteration into registers and release
        // it (the MMA issuer starts the next iteration's S), then dP chunk by
        // chunk, releasing it with the second chunk (the next dP), and form
        // dS into this iteration's dS buffer
        for (int u = J.i0; u < J.i1; ++u, ++n) {
          if (!mbar_wait_warp(BBAR(s_full), n & 1, wc, KERR_TIMEOUT_SOFTMAX)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const int kt = u < J.n0 ? u : J.w0 + (u - J.n0);
          // the dQ product two iterations back has read this iteration's dS buffer
          if (!mbar_wait_warp(BBAR(ds_free[0]) + 8 * (n & 1), ((n >> 1) & 1) ^ 1, wc, KERR_TIMEOUT_SOFTMAX)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          float sv[2][32];
          tmem_ld32f(tmem + lane_off + G::T1 + wg * 64, sv[0]);
          tmem_ld32f(tmem + lane_off + G::T1 + wg * 64 + 32, sv[1]);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(BBAR(s_free));
          if (!mbar_wait_warp(BBAR(dp_full), n & 1, wc, KERR_TIMEOUT_SOFTMAX)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint64_t sl2x2 = f2_pack(sl2, sl2);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float dv[32];
            tmem_ld32f(tmem + lane_off + G::T2 + wg * 64 + c * 32, dv);
            tmem_wait_ld();
            if (c == 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(BBAR(dp_free));
            }
            const int kb = kt * BWD_BN + wg * 64 + c * 32;
            uint32_t m = qvalid ? bits_range(0, qpos - kb + 1) : 0u;
            if (p.pass == BWD_SPARSE) m &= bits_range(0, p.sink - kb) | bits_range(qlo - kb, 32);
            // P = exp2(s * scale - lse) and dS = P (dP - D) on packed fp32 pairs
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(sv[c][e], sv[c][e + 1]), sl2x2, f2_pack(-qlse, -qlse)), a0, a1);
              const float p0 = ((m >> e) & 1u) ? fast_exp2(a0) : 0.f;
              const float p1 = ((m >> (e + 1)) & 1u) ? fast_exp2(a1) : 0.f;
              float d0, d1;
              f2_unpack(f2_mul(f2_pack(p0, p1), f2_sub(f2_pack(dv[e], dv[e + 1]), f2_pack(qd, qd))), d0, d1);
              pk[e >> 1] = pack_bf16x2(d0, d1);
            }
            __syncwarp();
            tmem_st16(tmem + lane_off + G::DS + (n & 1) * 64 + wg * 32 + c * 16, pk);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(BBAR(p_full));
        }
      } else
      for (int u = J.i0; u < J.i1; ++u, ++n) {
        // key-major: P^T(u) needs S^T(u) only; dS^T(u) then needs dP^T(u)
        if (!mbar_wait_warp(BBAR(s_full), n & 1, wc, KERR_TIMEOUT_SOFTMAX)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const int st = n & 1;
        const float* stats = reinterpret_cast<const float*>(base + G::STR_OFF + st * G::STAGE + 2 * G::TILE);
        // the query tile of this iteration
        const int ns = J.us1 - J.us0;
        const bool kdense = u >= ns;
        const int qt = kdense ? J.ud0 + (u - ns) : J.us0 + u;
        const int qbase = qt * p.R;
        // phase 1: P^T = exp2(S^T scale - lse) written over S^T in T1 (bf16),
        // 32 columns at a time; P^T is kept packed for phase 2
        const uint64_t sl2x2 = f2_pack(sl2, sl2);
        uint32_t pk[2][16];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col0 = wg * 64 + c * 32;
          float s[32];
          tmem_ld32f(tmem + lane_off + G::T1 + col0, s);
          tmem_wait_ld();
          // columns col0 .. col0+31 are rows rr0 + e of the tile (two runs of 16 when R = 16)
          uint32_t m;
          const int lo = kdense ? kfirst : klo, hi = kdense ? p.n_sel : khi;
          if (p.R >= 32) {
            const int b0 = qbase + (col0 & (p.R - 1));
            m = bits_range(lo - b0, hi - b0);
          } else {
            const uint32_t h16 = bits_range(lo - qbase, hi - qbase) & 0xffffu;
            m = h16 | (h16 << 16);
          }
          // the query rows' -lse come four at a time from the stage's stats
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 nl4 = *reinterpret_cast<const float4*>(stats + col0 + e);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int f = e + 2 * h;
              const uint64_t nl = h ? f2_pack(nl4.z, nl4.w) : f2_pack(nl4.x, nl4.y);
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(s[f], s[f + 1]), sl2x2, nl), a0, a1);
              const float p0 = ((m >> f) & 1u) ? fast_exp2(a0) : 0.f;
              const float p1 = ((m >> (f + 1)) & 1u) ? fast_exp2(a1) : 0.f;
              pk[c][f >> 1] = pack_bf16x2(p0, p1);
            }
          }
          __syncwarp();
          tmem_st16(tmem + lane_off + G::T1 + wg * 64 + c * 16, pk[c]);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BBAR(p_full));
        // phase 2: dS^T = P^T (dP^T - D) written over dP^T in T2 (bf16), from
        // the packed P^T (the bf16 values the dV product uses)
        if (!mbar_wait_warp(BBAR(dp_full), n & 1, wc, KERR_TIMEOUT_SOFTMAX)) {
          aborted = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int col0 = wg * 64 + c * 32;
          float dp[32];
          tmem_ld32f(tmem + lane_off + G::T2 + col0, dp);
          tmem_wait_ld();
          uint32_t dk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 dd4 = *reinterpret_cast<const float4*>(stats + 128 + col0 + e);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int f = e + 2 * h;
              const uint64_t dd = h ? f2_pack(dd4.z, dd4.w) : f2_pack(dd4.x, dd4.y);
              const uint32_t pp = pk[c][f >> 1];
              const uint64_t p2 = f2_pack(__uint_as_float(pp << 16), __uint_as_float(pp & 0xffff0000u));
              float d0, d1;
              f2_unpack(f2_mul(p2, f2_sub(f2_pack(dp[f], dp[f + 1]), dd)), d0, d1);
              dk[f >> 1] = pack_bf16x2(d0, d1);
            }
          }
          __syncwarp();
          tmem_st16(tmem + lane_off + G::T2 + wg * 64 + c * 16, dk);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BBAR(ds_full));
      }
      if (aborted) break;
      // ---- epilogue: this warpgroup's half of the accumulator columns ----
      if (!mbar_wait_warp(BBAR(acc_full), jobs & 1, wc, KERR_TIMEOUT_SOFTMAX)) break;
      tc_fence_after();
      constexpr int HALF = HD / 2;
      if constexpr (KM) {
        float a1[HALF], a2[HALF];
#pragma unroll
        for (int c = 0; c < HALF / 32; ++c) tmem_ld32f(tmem + lane_off + G::ACC1 + wg * HALF + c * 32, a1 + c * 32);
#pragma unroll
        for (int c = 0; c < HALF / 32; ++c) tmem_ld32f(tmem + lane_off + G::ACC2 + wg * HALF + c * 32, a2 + c * 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BBAR(acc_empty));
        if (key < p.S) {
          const long long o = (((long long)J.b * p.Hkv + J.g) * p.S + key) * HD + wg * HALF;
#pragma unroll
          for (int e = 0; e < HALF; e += 4) {
            red_add_v4(p.dv_acc + o + e, a1[e], a1[e + 1], a1[e + 2], a1[e + 3]);
            red_add_v4(p.dk_acc + o + e, a2[e], a2[e + 1], a2[e + 2], a2[e + 3]);
          }
        }
      } else {
        float a1[HALF];
#pragma unroll
        for (int c = 0; c < HALF / 32; ++c) tmem_ld32f(tmem + lane_off + G::ACC1 + wg * HALF + c * 32, a1 + c * 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BBAR(acc_empty));
        if (qvalid) {
          const int head = J.g * p.G + hh;
          const float sc = p.scaling;
          int out_row = -1;          // bf16 dq row, or -1
          float* dst32 = nullptr;    // fp32 dq_dn row (dense anchor rows)
          const float* add32 = nullptr;  // dense pass's dQ to add (windowed anchor rows)
          if (p.pass == BWD_DENSE) {
            const int i = J.tile * p.R + rr;
            if (i < p.n_anchor) dst32 = p.dq_dn + (((long long)J.b * p.H + head) * p.n_anchor + i) * HD + wg * HALF;
            else out_row = qpos;
          } else {
            out_row = qpos;
            if (p.n_anchor > 0 && qpos % p.gamma == 0 && qpos / p.gamma < p.n_anchor)
              add32 = p.dq_dn + (((long long)J.b * p.H + head) * p.n_anchor + qpos / p.gamma) * HD + wg * HALF;
          }
          if (dst32) {
#pragma unroll
            for (int e = 0; e < HALF; e += 4)
              *reinterpret_cast<float4*>(dst32 + e) = make_float4(a1[e] * sc, a1[e + 1] * sc, a1[e + 2] * sc, a1[e + 3] * sc);
          } else if (out_row >= 0) {
            __nv_bfloat16* dst = p.dq + (((long long)J.b * p.H + head) * p.S + out_row) * HD + wg * HALF;
#pragma unroll
            for (int e = 0; e < HALF; e += 8) {
              float v[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) v[k] = a1[e + k] * sc;
              if (add32) {
                const float4 x = *reinterpret_cast<const float4*>(add32 + e);
                const float4 y = *reinterpret_cast<const float4*>(add32 + e + 4);
                v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w;
                v[4] += y.x; v[5] += y.y; v[6] += y.z; v[7] += y.w;
              }
              uint4 w;
              w.x = pack_bf16x2(v[0], v[1]);
              w.y = pack_bf16x2(v[2], v[3]);
              w.z = pack_bf16x2(v[4], v[5]);
              w.w = pack_bf16x2(v[6], v[7]);
              *reinterpret_cast<uint4*>(dst + e) = w;
            }
          }
        }
      }
      ++jobs;
    }
  }
#undef BBAR
  // a key-major CTA never completes before the grid it may overlap (the
  // dense-row dQ launch), so work queued after this launch sees that grid done
  if (KM && threadIdx.x == 0) grid_dependency_wait();
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int HD, int KIND>
static cudaError_t launch_bwd_hd(const BackwardParams& p, int grid, bool dependent, cudaStream_t stream) {
  const int smem = KIND == BWD_KM ? BGeo<HD>::SMEM : BGeo<HD>::SMEM_QM;
  cudaError_t e = cudaFuncSetAttribute(bwd_kernel<HD, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(BWD_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, bwd_kernel<HD, KIND>, p);
}

cudaError_t launch_backward_dq(const BackwardParams& p, int head_dim, int grid, cudaStream_t stream) {
  return head_dim == 128 ? launch_bwd_hd<128, BWD_QM>(p, grid, false, stream)
                         : launch_bwd_hd<64, BWD_QM>(p, grid, false, stream);
}
cudaError_t launch_backward_dkdv(const BackwardParams& p, int head_dim, int grid, bool dependent, cudaStream_t stream) {
  return head_dim == 128 ? launch_bwd_hd<128, BWD_KM>(p, grid, dependent, stream)
                         : launch_bwd_hd<64, BWD_KM>(p, grid, dependent, stream);
}

}  // namespace dta

// ---------------------------------------------------------------------------
// C ABI: dta_backward_workspace_size / dta_backward
// ---------------------------------------------------------------------------
#include <string.h>

#include "delta_attention_b200.h"
#include "dta_internal.h"

namespace {

constexpr size_t kBwdHeader = 256;  // job counters (ints 0, 2, 3), error word (int 1, as dta_check_workspace reads)
constexpr int kBwdChunkIters = 64;  // query tiles per key-major job

inline size_t bwd_align(size_t x) { return (x + 255) / 256 * 256; }

struct BwdLayout {
  int s_p, n_anchor, n_sel, n_ktiles;
  size_t off_chunk, off_gsp, off_gdn, off_qsel, off_dsp, off_ddn, off_dqdn, off_dk, off_dv, total;
};

int backward_layout(const dta_backward_args* a, BwdLayout* L) {
  if (!a || a->abi_version != DTA_ABI_VERSION) return DTA_ERR_INVALID_ARG;
  if (a->batch <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->seq_len <= 0) return DTA_ERR_SHAPE;
  if (a->head_dim != 64 && a->head_dim != 128) return DTA_ERR_HEAD_DIM;
  if (a->n_heads % a->n_kv_heads != 0) return DTA_ERR_SHAPE;
  const int G = a->n_heads / a->n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return DTA_ERR_SHAPE;
  if (a->window < 0 || a->sink < 0 || a->q_block <= 0 || a->gamma <= 0) return DTA_ERR_INVALID_ARG;
  if (!(a->delta_grad_scale == a->delta_grad_scale)) return DTA_ERR_INVALID_ARG;  // NaN
  const int s = a->seq_len;
  const int cut_n = s % a->gamma + (a->gamma > 128 ? a->gamma : 128);
  const int s_p = s - cut_n;
  if (s_p <= 0 || s_p % a->gamma != 0) return DTA_ERR_GAMMA;
  L->s_p = s_p;
  L->n_anchor = s_p / a->gamma;
  L->n_sel = L->n_anchor + cut_n;
  L->n_ktiles = (s + dta::BWD_BN - 1) / dta::BWD_BN;
  const size_t B = a->batch, H = a->n_heads, Hkv = a->n_kv_heads, d = a->head_dim;
  size_t off = kBwdHeader;
  L->off_chunk = off; off += bwd_align((size_t)(L->n_ktiles + 1) * 4);
  L->off_gsp = off;   off += bwd_align(B * s_p * H * d * 2);
  L->off_gdn = off;   off += bwd_align(B * L->n_sel * H * d * 2);
  L->off_qsel = off;  off += bwd_align(B * H * L->n_sel * d * 2);
  L->off_dsp = off;   off += bwd_align(B * H * s * 4);
  L->off_ddn = off;   off += bwd_align(B * H * L->n_sel * 4);
  L->off_dqdn = off;  off += bwd_align(B * H * L->n_anchor * d * 4);
  L->off_dk = off;    off += bwd_align(B * Hkv * s * d * 4);
  L->off_dv = off;    off += bwd_align(B * Hkv * s * d * 4);
  L->total = off;
  return DTA_OK;
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
inline bool st16(long long s) { return s > 0 && (s * 2) % 16 == 0; }

}  // namespace

extern "C" {

size_t dta_backward_workspace_size(const dta_backward_args* a) {
  BwdLayout L;
  if (backward_layout(a, &L) != DTA_OK) return 0;
  return L.total;
}

int dta_backward(const dta_backward_args* a, void* stream_) {
  BwdLayout L;
  int st = backward_layout(a, &L);
  if (st != DTA_OK) return st;
  if (!a->q || !a->k || !a->v || !a->out || !a->grad_out || !a->anchor_delta || !a->lse_sparse || !a->lse_dense ||
      !a->grad_q || !a->grad_k || !a->grad_v)
    return DTA_ERR_INVALID_ARG;
  if (!a->workspace || a->workspace_bytes < L.total || !al16(a->workspace)) return DTA_ERR_WORKSPACE;
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->out) || !al16(a->grad_out) || !al16(a->anchor_delta) ||
      !al16(a->grad_q) || !al16(a->grad_k) || !al16(a->grad_v) || ((uintptr_t)a->lse_sparse & 3u) ||
      ((uintptr_t)a->lse_dense & 3u))
    return DTA_ERR_ALIGNMENT;
  if (!st16(a->q_stride_s) || !st16(a->q_stride_h) || !st16(a->q_stride_b) || !st16(a->k_stride_s) ||
      !st16(a->k_stride_h) || !st16(a->k_stride_b) || !st16(a->v_stride_s) || !st16(a->v_stride_h) ||
      !st16(a->v_stride_b))
    return DTA_ERR_STRIDE;
  if (a->error_word && ((uintptr_t)a->error_word & 3u) != 0) return DTA_ERR_ALIGNMENT;
  if (a->wait_cycles < 0) return DTA_ERR_INVALID_ARG;
  int sms = 0;
  if ((st = dta::check_device(&sms)) != DTA_OK) return st;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int B = a->batch, H = a->n_heads, Hkv = a->n_kv_heads, S = a->seq_len, d = a->head_dim;
  const int G = H / Hkv, R = 128 / G;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  auto at = [&](size_t off) { return ws + off; };
  __nv_bfloat16* g_sp = reinterpret_cast<__nv_bfloat16*>(at(L.off_gsp));
  __nv_bfloat16* g_dn = reinterpret_cast<__nv_bfloat16*>(at(L.off_gdn));
  __nv_bfloat16* q_sel = reinterpret_cast<__nv_bfloat16*>(at(L.off_qsel));
  float* d_sp = reinterpret_cast<float*>(at(L.off_dsp));
  float* d_dn = reinterpret_cast<float*>(at(L.off_ddn));
  int* chunk_base = reinterpret_cast<int*>(at(L.off_chunk));

  dta::BackwardParams p;
  memset(&p, 0, sizeof(p));
  p.B = B; p.H = H; p.Hkv = Hkv; p.G = G; p.R = R; p.S = S;
  p.s_p = L.s_p; p.n_anchor = L.n_anchor; p.n_sel = L.n_sel;
  p.gamma = a->gamma; p.window = a->window; p.sink = a->sink; p.qblock = a->q_block;
  p.scaling = a->scaling;
  p.scale_log2 = a->scaling * 1.4426950408889634f;
  p.lse_sp = a->lse_sparse;
  p.lse_dn = a->lse_dense;
  p.d_sp = d_sp;
  p.d_dn = d_dn;
  p.dq = reinterpret_cast<__nv_bfloat16*>(a->grad_q);
  p.dq_dn = reinterpret_cast<float*>(at(L.off_dqdn));
  p.dk_acc = reinterpret_cast<float*>(at(L.off_dk));
  p.dv_acc = reinterpret_cast<float*>(at(L.off_dv));
  p.n_ktiles = L.n_ktiles;
  p.chunk_iters = kBwdChunkIters;
  p.chunk_base = chunk_base;
  p.error = a->error_word ? a->error_word : reinterpret_cast<int*>(ws) + 1;
  p.wait_cycles = a->wait_cycles > 0 ? a->wait_cycles : dta::kWaitTimeoutCycles;
  if ((st = dta::encode_4d(&p.tm_q, a->q, d, S, H, B, a->q_stride_s, a->q_stride_h, a->q_stride_b, R, G)) != DTA_OK ||
      (st = dta::encode_4d(&p.tm_qsel, q_sel, d, L.n_sel, H, B, d, (long long)L.n_sel * d, (long long)H * L.n_sel * d, R,
                           G)) != DTA_OK ||
      (st = dta::encode_4d(&p.tm_k, a->k, d, S, Hkv, B, a->k_stride_s, a->k_stride_h, a->k_stride_b, dta::BWD_BN, 1)) !=
          DTA_OK ||
      (st = dta::encode_4d(&p.tm_v, a->v, d, S, Hkv, B, a->v_stride_s, a->v_stride_h, a->v_stride_b, dta::BWD_BN, 1)) !=
          DTA_OK ||
      (st = dta::encode_4d(&p.tm_gsp, g_sp, d, L.s_p, H, B, d, (long long)L.s_p * d, (long long)H * L.s_p * d, R, G)) !=
          DTA_OK ||
      (st = dta::encode_4d(&p.tm_gdn, g_dn, d, L.n_sel, H, B, d, (long long)L.n_sel * d, (long long)H * L.n_sel * d, R, G)) !=
          DTA_OK)
    return st;
  // the key-major launch's job count (the device plan computes the same table)
  int total_chunks = 0;
  for (int kt = 0; kt < L.n_ktiles; ++kt) {
    const dta::KeyTileList K = dta::bwd_key_tile_list(kt, S, L.s_p, L.n_anchor, L.n_sel, a->gamma, a->window, a->sink,
                                                      a->q_block, R);
    total_chunks += ((K.us1 - K.us0) + (K.ud1 - K.ud0) + kBwdChunkIters - 1) / kBwdChunkIters;
  }
  p.total_chunks = total_chunks;

  cudaError_t e;
  // counters and error word, the dK / dV accumulators
  if ((e = cudaMemsetAsync(ws, 0, kBwdHeader, stream)) != cudaSuccess) return dta::fail_cuda(e);
  if ((e = cudaMemsetAsync(at(L.off_dk), 0, L.total - L.off_dk, stream)) != cudaSuccess) return dta::fail_cuda(e);
  if ((e = dta::launch_backward_prep(reinterpret_cast<const __nv_bfloat16*>(a->q), a->q_stride_b, a->q_stride_h,
                                     a->q_stride_s, reinterpret_cast<const __nv_bfloat16*>(a->out),
                                     reinterpret_cast<const __nv_bfloat16*>(a->grad_out), a->anchor_delta, g_sp, g_dn,
                                     q_sel, d_sp, d_dn, B, H, S, d, L.s_p, L.n_anchor, L.n_sel, a->gamma,
                                     a->delta_grad_scale, stream)) != cudaSuccess)
    return dta::fail_cuda(e);
  if ((e = dta::launch_backward_plan(chunk_base, L.n_ktiles, S, L.s_p, L.n_anchor, L.n_sel, a->gamma, a->window,
                                     a->sink, a->q_block, R, kBwdChunkIters, stream)) != cudaSuccess)
    return dta::fail_cuda(e);
  // dQ of the dense rows first (its longest job spans every key tile), the
  // key-major dK / dV launch queued behind it as a programmatic dependent
  // launch (independent of its output; its CTAs take SMs as the dense grid's
  // finish), then dQ of the windowed rows, which adds the dense rows' dQ at
  // each anchor row
  dta::BackwardParams q = p;
  q.counter = reinterpret_cast<int*>(ws) + 2;
  q.pass = dta::BWD_DENSE;
  q.n_qtiles = (L.n_sel + R - 1) / R;
  q.n_jobs = q.n_qtiles * B * Hkv;
  if ((e = dta::launch_backward_dq(q, d, q.n_jobs < sms ? q.n_jobs : sms, stream)) != cudaSuccess)
    return dta::fail_cuda(e);
  {
    dta::BackwardParams k = p;
    k.counter = reinterpret_cast<int*>(ws) + 0;
    k.n_jobs = total_chunks * B * Hkv;
    if (k.n_jobs > 0 && (e = dta::launch_backward_dkdv(k, d, k.n_jobs < sms ? k.n_jobs : sms, true, stream)) !=
                            cudaSuccess)
      return dta::fail_cuda(e);
  }
  q.counter = reinterpret_cast<int*>(ws) + 3;
  q.pass = dta::BWD_SPARSE;
  q.n_qtiles = (L.s_p + R - 1) / R;
  q.n_jobs = q.n_qtiles * B * Hkv;
  if ((e = dta::launch_backward_dq(q, d, q.n_jobs < sms ? q.n_jobs : sms, stream)) != cudaSuccess)
    return dta::fail_cuda(e);
  const long long n = (long long)B * Hkv * S * d;
  if ((e = dta::launch_backward_finalize(p.dk_acc, p.dv_acc, reinterpret_cast<__nv_bfloat16*>(a->grad_k),
                                         reinterpret_cast<__nv_bfloat16*>(a->grad_v), n, a->scaling, stream)) !=
      cudaSuccess)
    return dta::fail_cuda(e);
  return DTA_OK;
}

}  // extern "C"
