// Decode attention on sm_100a: one query row per (batch, head) over a KV cache.
//
// Split-K over the cache: CTA (chunk, batch x kv-group, key set) streams its
// chunk of K and V through shared memory once, serves every query head of the
// GQA group with tensor-core products, and forms an unnormalised partial
// (max, sum, o[d]) for its key set: DENSE (every key) or SPARSE (the first
// `sink` keys plus the last `window` keys; delta_attention/llama.py:538-550).
// The dense set's partials go to global memory and a merge kernel combines
// them with the log-sum-exp rule; it is a programmatic dependent launch
// (DTA_DEC_PDL_MERGE), so its CTAs become resident while the partials run and
// wait on the device for them.  The sparse set's chunks tile [0, sink) and
// [n - window, n) exactly; when they fit one thread-block cluster per (batch,
// group), the cluster merges them through distributed shared memory and a
// sparse-only step is a single launch (DTA_DEC_SPARSE_CLUSTER).  An anchor
// step of delta decode (delta_attention/llama.py:552-634) launches the dense
// grid, then the sparse grid (which re-reads the sink and window from L2),
// then the merge; a non-anchor step launches only the sparse grid.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "dta_ptx.cuh"
#include "dta_decode.h"

// 0: plain merge launch; 1: programmatic dependent merge on sparse-only calls;
// 2: on every call
#ifndef DTA_DEC_PDL_MERGE
#define DTA_DEC_PDL_MERGE 2
#endif
// 1: the sparse set merges in-cluster (one launch for a sparse-only step)
#ifndef DTA_DEC_SPARSE_CLUSTER
#define DTA_DEC_SPARSE_CLUSTER 1
#endif

namespace dta {

constexpr int DEC_THREADS = 128;

// The live key count and whether every key is sparse: host values, or (DEVN,
// a separate kernel instance) read from the device count for CUDA-graph
// replays, so the host-count instance is free of the device-count logic.
template <bool DEVN>
__device__ __forceinline__ int dec_n_keys(const DecodeParams& p) {
  if constexpr (DEVN) return min(max(*p.n_keys_dev, 1), p.n_keys);
  return p.n_keys;
}
template <bool DEVN>
__device__ __forceinline__ bool dec_all_sparse(const DecodeParams& p, int n) {
  if constexpr (DEVN) return (long long)n <= (long long)p.sink + p.window;
  return p.all_sparse != 0;
}

// Key range [k0, k1) of launched chunk x of the sparse set with n live keys:
// [0, sink) and then [n - window, n) tiled from each range's first key, or
// [0, n) when every key is sparse.  An empty range leaves an empty partial.
__device__ __forceinline__ void dec_sparse_range(const DecodeParams& p, const DecodeSet& S, bool all_sparse, int n,
                                                 int x, int& k0, int& k1) {
  if (all_sparse) {
    k0 = x * S.chunk;
    k1 = min(k0 + S.chunk, n);
  } else if (x >= S.n_sink_chunks) {
    k0 = n - p.window + (x - S.n_sink_chunks) * S.chunk;
    k1 = min(k0 + S.chunk, n);
  } else {
    k0 = x * S.chunk;
    k1 = min(k0 + S.chunk, p.sink);
  }
}

// Kinds of partial launch: the dense set (partials to the merge kernel), the
// sparse set (likewise), the sparse set merged in-cluster.
constexpr int DEC_DENSE = 0, DEC_SPARSE = 1, DEC_SPARSE_CLU = 2;

// ---------------------------------------------------------------------------
// Tensor-core partial kernel.  CTA = (chunk of S.chunk keys, batch x KV
// group, key set), 4 warps.  The chunk's K and V rows stream through shared
// memory in 64-key stages (cp.async, 16-byte chunks XOR-swizzled by row so
// ldmatrix is conflict-free, DEC_NSTAGE stages in flight).  Warp w owns keys
// [16w, 16w + 16) of every stage and runs, per stage, S = Q K^T and O += P V
// with mma.sync m16n8k16 (bf16 in, fp32 accumulate): the M = 16 rows are the
// G <= 8 query heads of the group (rows >= G are zero), N runs over keys for
// S and over head dims for O, and the S accumulator fragments become the P
// operand fragments in registers.  An online softmax (running max and sum per
// head, exact rescale) runs on the fragments; the four warps' states are
// merged once per chunk.  KIND selects the key set and its chunking: the
// dense set (every key, long chunks) or the sparse set (sink + window, short
// chunks holding only sparse keys); an anchor step launches both, and the
// sparse launch re-reads the sink and window keys (from L2).
// ---------------------------------------------------------------------------
constexpr int DEC_STAGE = 64;  // keys per shared-memory stage
#ifndef DTA_DEC_NSTAGE
#define DTA_DEC_NSTAGE 3
#endif
constexpr int DEC_NSTAGE = DTA_DEC_NSTAGE;  // stages in flight

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D = A B + D, m16n8k16, A row-major bf16, B column-major bf16, fp32 accumulate.
// Rows 8..15 of A are zero here, so a1 = a3 = 0.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// DEC_SPARSE_CLU: the grid's x extent is one thread-block cluster per (batch,
// group) and the chunks' partials merge through distributed shared memory
// instead of the merge kernel (the sparse set when its chunks fit one cluster).
template <int HD, bool DEVN, int KIND>
__global__ void __launch_bounds__(DEC_THREADS) decode_mma_kernel(const __grid_constant__ DecodeParams p) {
  constexpr bool CLU = KIND == DEC_SPARSE_CLU;
  constexpr int CH = HD / 8;                  // 16-byte chunks per row
  constexpr int ROWB = HD * 2;                // bytes per K/V row
  constexpr int STAGE_BYTES = DEC_STAGE * ROWB;
  constexpr int NT = HD / 8;                  // n-tiles of O
  extern __shared__ __align__(128) uint8_t dsm[];
  // layout: [DEC_NSTAGE stages] x {K, V} x STAGE_BYTES; reused for the merge after the loop
  const uint32_t sbase = smem_u32(dsm);

  // lets a programmatic dependent merge launch start its CTAs now; they wait
  // in griddepcontrol.wait for this grid's completion and its memory flush
  grid_dependents_launch();
  const DecodeSet& S = p.set[KIND == DEC_DENSE ? 0 : 1];
  const int n_live = dec_n_keys<DEVN>(p);
  int k0, k1;
  if constexpr (KIND == DEC_DENSE) {
    k0 = blockIdx.x * S.chunk;
    k1 = min(k0 + S.chunk, n_live);
  } else {
    dec_sparse_range(p, S, dec_all_sparse<DEVN>(p, n_live), n_live, blockIdx.x, k0, k1);
  }
  const int bg = blockIdx.y;
  const int b = bg / p.Hkv, g = bg - (bg / p.Hkv) * p.Hkv;
  const int G = p.G;
  // (a chunk past the live keys of a device count has none and leaves an empty partial)
  const int nk = (KIND == DEC_DENSE && !DEVN) ? k1 - k0 : max(k1 - k0, 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, cq = lane & 3;  // fragment row (= head) and column pair
  float* part0 = S.partials + ((long long)(b * p.H + g * G) * S.n_launched + blockIdx.x) * (4 + HD);
  const long long hstride = (long long)S.n_launched * (4 + HD);

  // Q fragments (A operand rows = heads): a0 = q[gr][16kk + 2cq, +1], a2 = [.. + 8]
  uint32_t qa[HD / 16][2];
  {
    const bool hv = gr < G;
    const __nv_bfloat16* qp = p.q + (long long)b * p.q_sb + (long long)(g * G + (hv ? gr : 0)) * p.q_sh;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      qa[kk][0] = hv ? *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 2 * cq) : 0u;
      qa[kk][1] = hv ? *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 8 + 2 * cq) : 0u;
    }
  }
  const __nv_bfloat16* kb = p.k + (long long)b * p.k_sb + (long long)g * p.k_sh;
  const __nv_bfloat16* vb = p.v + (long long)b * p.v_sb + (long long)g * p.v_sh;
  const int n_stages = (nk + DEC_STAGE - 1) / DEC_STAGE;
  auto load_stage = [&](int s) {
    const uint32_t kdst = sbase + (uint32_t)(s % DEC_NSTAGE) * 2 * STAGE_BYTES;
    const uint32_t vdst = kdst + STAGE_BYTES;
    const int j0 = s * DEC_STAGE;
    for (int idx = threadIdx.x; idx < DEC_STAGE * CH; idx += DEC_THREADS) {
      const int r = idx / CH, ch = idx - (idx / CH) * CH;
      const int j = j0 + r;
      const bool ok = j < nk;
      const long long key = k0 + (ok ? j : 0);
      const uint32_t off = (uint32_t)(r * ROWB + ((ch ^ (r & 7)) << 4));
      cp_async_16(kdst + off, kb + key * p.k_ss + ch * 8, ok ? 16u : 0u);
      cp_async_16(vdst + off, vb + key * p.v_ss + ch * 8, ok ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float m_run = -INFINITY, l_run = 0.f;  // head gr (rows >= G carry nothing)
  float o[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  const float sl2 = p.scale_log2;

  // DEC_NSTAGE - 1 stages ahead; one commit group per iteration (empty past
  // the end) keeps "stage s complete" at wait_group DEC_NSTAGE - 1
  for (int s = 0; s < DEC_NSTAGE - 1; ++s) {
    if (s < n_stages) load_stage(s);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int s = 0; s < n_stages; ++s) {
    if (s + DEC_NSTAGE - 1 < n_stages) load_stage(s + DEC_NSTAGE - 1);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(DEC_NSTAGE - 1) : "memory");
    __syncthreads();
    const uint32_t ks = sbase + (uint32_t)(s % DEC_NSTAGE) * 2 * STAGE_BYTES;
    const uint32_t vs = ks + STAGE_BYTES;
    const int r0 = warp * 16;  // this warp's first key row in the stage
    // ---- S = Q K^T for 16 keys (two n-tiles of 8 keys) ----
    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int r = r0 + (mi >> 1) * 8 + rr;  // matrices 0,1: keys 0-7; 2,3: keys 8-15
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const int ch = 2 * kk + (mi & 1);
        uint32_t b00, b01, b10, b11;
        ldsm_x4(ks + (uint32_t)(r * ROWB + ((ch ^ (r & 7)) << 4)), b00, b01, b10, b11);
        mma_16816(sacc[0], qa[kk][0], qa[kk][1], b00, b01);
        mma_16816(sacc[1], qa[kk][0], qa[kk][1], b10, b11);
      }
    }
    // ---- online softmax on row gr: keys 2cq, 2cq+1 (tile 0) and 8+2cq, 9+2cq (tile 1) ----
    float sv[4] = {sacc[0][0] * sl2, sacc[0][1] * sl2, sacc[1][0] * sl2, sacc[1][1] * sl2};
    const int jb = s * DEC_STAGE + r0;  // chunk-local key of fragment column 0
    const int jk[4] = {jb + 2 * cq, jb + 2 * cq + 1, jb + 8 + 2 * cq, jb + 9 + 2 * cq};
#pragma unroll
    for (int e = 0; e < 4; ++e) sv[e] = jk[e] < nk ? sv[e] : -INFINITY;
    float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_new);
    float pv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pv[e] = fast_exp2(sv[e] - m_use);
    l_run = l_run * alpha + (pv[0] + pv[1]) + (pv[2] + pv[3]);
    m_run = m_new;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      o[t][0] *= alpha;
      o[t][1] *= alpha;
    }
    const uint32_t pa0 = pack_bf16x2(pv[0], pv[1]);
    const uint32_t pa2 = pack_bf16x2(pv[2], pv[3]);
    // ---- O += P V: B fragments by transposed ldmatrix, two n-tiles per load ----
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int r = r0 + (mi & 1) * 8 + rr;  // matrices 0,2: keys 0-7; 1,3: keys 8-15
#pragma unroll
      for (int t = 0; t < NT; t += 2) {
        const int ch = t + (mi >> 1);
        uint32_t b00, b01, b10, b11;
        ldsm_x4_t(vs + (uint32_t)(r * ROWB + ((ch ^ (r & 7)) << 4)), b00, b01, b10, b11);
        mma_16816(o[t], pa0, pa2, b00, b01);
        mma_16816(o[t + 1], pa0, pa2, b10, b11);
      }
    }
    __syncthreads();  // the stage may be refilled
  }
  // ---- merge the four warps: row sums over the 4 lanes of a row, then over warps ----
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  float* red_o = reinterpret_cast<float*>(dsm);                       // [4][8][HD]
  float* red_ml = red_o + 4 * 8 * HD;                                 // [4][2][8]
  if (cq == 0) {
    red_ml[(warp * 2 + 0) * 8 + gr] = m_run;
    red_ml[(warp * 2 + 1) * 8 + gr] = l_run;
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red_o[(warp * 8 + gr) * HD + t * 8 + 2 * cq] = o[t][0];
    red_o[(warp * 8 + gr) * HD + t * 8 + 2 * cq + 1] = o[t][1];
  }
  __syncthreads();
  float* cl_o = red_ml + 4 * 2 * 8;  // CLU: this chunk's partial [8][HD], then (m, l) [2][8]
  float* cl_ml = cl_o + 8 * HD;
  for (int idx = threadIdx.x; idx < G * HD; idx += DEC_THREADS) {
    const int h = idx / HD, t = idx - (idx / HD) * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_ml[(w * 2) * 8 + h]);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float m = red_ml[(w * 2) * 8 + h];
        if (m == -INFINITY) continue;
        const float sc = fast_exp2(m - M);
        O += red_o[(w * 8 + h) * HD + t] * sc;
        L += red_ml[(w * 2 + 1) * 8 + h] * sc;
      }
    }
    if constexpr (CLU) {
      cl_o[h * HD + t] = O;
      if (t == 0) {
        cl_ml[h] = M;
        cl_ml[8 + h] = L;
      }
    } else {
      float* part = part0 + h * hstride;
      part[4 + t] = O;
      if (t == 0) {
        part[0] = M;
        part[1] = L;
      }
    }
  }
  if constexpr (CLU) {
    // every chunk's partial is in its CTA's shared memory; the cluster's CTAs
    // split the group's G * HD outputs and merge the chunks in rank (= chunk)
    // order with the log-sum-exp rule of the merge kernel
    __syncwarp();
    cluster_sync();
    const int nct = (int)cluster_nctarank(), rank = (int)cluster_ctarank();
    const uint32_t o_addr = smem_u32(cl_o), ml_addr = smem_u32(cl_ml);
    // host key count with n <= sink + window: the sparse set is the dense set too
    __nv_bfloat16* dense_dst = (!DEVN && p.all_sparse) ? p.dense_out : nullptr;
    for (int idx = rank * DEC_THREADS + threadIdx.x; idx < G * HD; idx += nct * DEC_THREADS) {
      const int h = idx / HD, t = idx - (idx / HD) * HD;
      float mv[DEC_CLUSTER_MAX];
#pragma unroll
      for (int r = 0; r < DEC_CLUSTER_MAX; ++r)
        mv[r] = r < nct ? ld_dsmem_f32(dsmem_addr(ml_addr + 4u * h, r)) : -INFINITY;
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < DEC_CLUSTER_MAX; ++r) M = fmaxf(M, mv[r]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
        float lv[DEC_CLUSTER_MAX], ov[DEC_CLUSTER_MAX];
#pragma unroll
        for (int r = 0; r < DEC_CLUSTER_MAX; ++r) {
          const bool live = mv[r] != -INFINITY;
          lv[r] = live ? ld_dsmem_f32(dsmem_addr(ml_addr + 4u * (8 + h), r)) : 0.f;
          ov[r] = live ? ld_dsmem_f32(dsmem_addr(o_addr + 4u * (h * HD + t), r)) : 0.f;
        }
#pragma unroll
        for (int r = 0; r < DEC_CLUSTER_MAX; ++r) {
          if (mv[r] == -INFINITY) continue;
          const float w = fast_exp2(mv[r] - M);
          L += lv[r] * w;
          O += ov[r] * w;
        }
      }
      const __nv_bfloat16 o16 = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
      const long long off = ((long long)b * p.H + g * G + h) * HD + t;
      if (p.sparse_out) p.sparse_out[off] = o16;
      if (dense_dst) dense_dst[off] = o16;
    }
    __syncwarp();
    cluster_sync();  // no CTA exits while a peer may still read its partial
  }
}

// Merge the partials of every launched chunk of a key set: grid (B*H), block
// HD.  One pass with a running rescale: each tile of DEC_MERGE_TILE partials
// issues all its loads (the (m, l) pair, the same address for every thread,
// and the thread's column of o) before any is used, so a key set of up to
// DEC_MERGE_TILE chunks costs one round trip to L2.
constexpr int DEC_MERGE_TILE = 16;

template <int HD, bool DEVN>
__global__ void decode_merge_kernel(const __grid_constant__ DecodeParams p) {
  const int bh = blockIdx.x;
  const int t = threadIdx.x;
  grid_dependency_wait();  // no-op unless launched as a programmatic dependent
  for (int out = 0; out < 2; ++out) {
    __nv_bfloat16* dst = out == 0 ? p.dense_out : p.sparse_out;
    if (!dst || (out == 1 && p.sparse_merged)) continue;
    // with n <= sink + window the two key sets coincide: both outputs come
    // from the sparse set's partials (host key count; with a device count the
    // dense output keeps the dense set, which covers the same keys)
    const DecodeSet& S = p.set[DEVN ? out : (out == 1 || p.all_sparse) ? 1 : 0];
    const float* base = S.partials + (long long)bh * S.n_launched * (4 + HD);
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int x0 = 0; x0 < S.n_launched; x0 += DEC_MERGE_TILE) {
      float mv[DEC_MERGE_TILE], lv[DEC_MERGE_TILE], ov[DEC_MERGE_TILE];
#pragma unroll
      for (int u = 0; u < DEC_MERGE_TILE; ++u) {
        const int x = x0 + u;
        if (x < S.n_launched) {
          const float* part = base + (long long)x * (4 + HD);
          const float2 ml = *reinterpret_cast<const float2*>(part);
          mv[u] = ml.x;
          lv[u] = ml.y;
          ov[u] = part[4 + t];
        } else {
          mv[u] = -INFINITY;
          lv[u] = ov[u] = 0.f;
        }
      }
      float mt = M;
#pragma unroll
      for (int u = 0; u < DEC_MERGE_TILE; ++u) mt = fmaxf(mt, mv[u]);
      if (mt == -INFINITY) continue;
      if (M != -INFINITY) {
        const float sc = fast_exp2(M - mt);
        L *= sc;
        O *= sc;
      }
#pragma unroll
      for (int u = 0; u < DEC_MERGE_TILE; ++u) {
        if (mv[u] == -INFINITY) continue;
        const float w = fast_exp2(mv[u] - mt);
        L += lv[u] * w;
        O += ov[u] * w;
      }
      M = mt;
    }
    const float o = L > 0.f ? O / L : 0.f;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    dst[((long long)b * p.H + h) * HD + t] = __float2bfloat16_rn(o);
  }
}

// Sets the CLU kernel's launch attributes for a cluster of `nct` CTAs on the
// current device (the dynamic shared memory, and the non-portable cluster
// sizes above 8).
template <int HD, bool DEVN>
static cudaError_t cluster_attrs(int nct, int smem) {
  auto kernel = decode_mma_kernel<HD, DEVN, DEC_SPARSE_CLU>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess && nct > 8) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e;
}

// Whether `nct` CTAs of the CLU kernel fit one cluster on the current device
// (cudaOccupancyMaxActiveClusters > 0), cached per device and size.
template <int HD, bool DEVN>
static bool cluster_fits(int nct, int smem) {
  constexpr int kDevices = 64;
  static std::mutex mu;
  static int fits[kDevices][DEC_CLUSTER_MAX + 1] = {};  // 0 unknown, 1 yes, 2 no
  if (nct < 1 || nct > DEC_CLUSTER_MAX) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevices) {
    (void)cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (fits[dev][nct] == 0) {
    int n = 0;
    cudaError_t e = cluster_attrs<HD, DEVN>(nct, smem);
    if (e == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(nct);
      cfg.blockDim = dim3(DEC_THREADS);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = nct;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      e = cudaOccupancyMaxActiveClusters(&n, decode_mma_kernel<HD, DEVN, DEC_SPARSE_CLU>, &cfg);
    }
    if (e != cudaSuccess) (void)cudaGetLastError();  // a refused size is not an error of the call
    fits[dev][nct] = (e == cudaSuccess && n > 0) ? 1 : 2;
  }
  return fits[dev][nct] == 1;
}

template <int HD, bool DEVN>
static cudaError_t launch_hd(const DecodeParams& p_in, cudaStream_t stream) {
  constexpr int smem = DEC_NSTAGE * 2 * DEC_STAGE * HD * 2;
  static_assert(smem >= (4 * 8 * HD + 4 * 2 * 8 + 8 * HD + 2 * 8) * 4, "merge buffers fit in the stage buffers");
  DecodeParams p = p_in;
  const bool dense_set = p.dense_out && !p.all_sparse;
  const bool sparse_set = p.sparse_out || p.all_sparse;
  const int nct = p.set[1].n_launched;
  const bool clu = DTA_DEC_SPARSE_CLUSTER && sparse_set && cluster_fits<HD, DEVN>(nct, smem);
  p.sparse_merged = clu ? 1 : 0;
  cudaError_t e;
  if (dense_set) {
    auto kernel = decode_mma_kernel<HD, DEVN, DEC_DENSE>;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kernel<<<dim3(p.set[0].n_launched, p.B * p.Hkv), DEC_THREADS, smem, stream>>>(p);
  }
  if (sparse_set && clu) {
    if ((e = cluster_attrs<HD, DEVN>(nct, smem)) != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nct, p.B * p.Hkv);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = nct;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_mma_kernel<HD, DEVN, DEC_SPARSE_CLU>, p);
    if (e != cudaSuccess) return e;
  } else if (sparse_set) {
    auto kernel = decode_mma_kernel<HD, DEVN, DEC_SPARSE>;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kernel<<<dim3(nct, p.B * p.Hkv), DEC_THREADS, smem, stream>>>(p);
  }
  // the merge kernel: the dense set's output, and the sparse set's unless merged in-cluster
  if (dense_set || !clu) {
    const bool pdl = DTA_DEC_PDL_MERGE == 2 || (DTA_DEC_PDL_MERGE == 1 && !dense_set);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.B * p.H);
    cfg.blockDim = dim3(HD);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, decode_merge_kernel<HD, DEVN>, p);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeParams& p, int head_dim, cudaStream_t stream) {
  if (head_dim == 128) return p.n_keys_dev ? launch_hd<128, true>(p, stream) : launch_hd<128, false>(p, stream);
  return p.n_keys_dev ? launch_hd<64, true>(p, stream) : launch_hd<64, false>(p, stream);
}

}  // namespace dta
