// Decode attention on sm_100a: one query row per (batch, head) over a KV cache.
//
// Split-K over the cache: CTA (chunk, batch x kv-group) reads its chunk of K
// and V exactly once with 16-byte-coalesced loads, serving every query head of
// the GQA group, and writes an unnormalised partial (max, sum, o[d]) for the
// DENSE key set and, when the chunk touches it, for the SPARSE key set (the
// first `sink` keys plus the last `window` keys; delta_attention/llama.py:538-550).
// A merge kernel combines the partials with the log-sum-exp rule.  An anchor
// step of delta decode (delta_attention/llama.py:552-634) therefore gets both
// its dense and its sparse row from one pass over the cache; a non-anchor step
// launches only the chunks that intersect the sparse key set.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "dta_ptx.cuh"
#include "dta_decode.h"

namespace dta {

constexpr int DEC_THREADS = 128;

__device__ __forceinline__ bool dec_sparse_key(const DecodeParams& p, int j) {
  return p.all_sparse || j < p.sink || j >= p.n_keys - p.window;
}

__device__ __forceinline__ int dec_chunk_of_block(const DecodeParams& p, int x) {
  if (p.want_dense || p.all_sparse) return x;
  return x < p.n_sink_chunks ? x : p.first_window_chunk + (x - p.n_sink_chunks);
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}

// One CTA per (chunk, batch x KV group), one pass over the chunk: each warp
// streams its own key steps (KPW keys per step, DEC_U steps per batch of
// loads, K and V of a batch requested before any arithmetic) and keeps an
// online softmax -- running max, sum and unnormalised o -- for the dense and
// the sparse key set.  The four warps' states are merged once at the end.
constexpr int DEC_U = 2;
template <int HD, int G>
__global__ void __launch_bounds__(DEC_THREADS, 3) decode_partial_kernel(const __grid_constant__ DecodeParams p) {
  constexpr int SUB = HD / 16;   // lanes per key in the QK product (16 dims each)
  constexpr int KPW = 32 / SUB;  // keys per warp step
  constexpr int DPL = HD / 32;   // dims per lane in the PV product
  constexpr int NW = DEC_THREADS / 32;
  __shared__ float wsc[NW][KPW][G];       // one step's scores, broadcast to the warp
  __shared__ float red_o[NW][G][HD];      // per-warp o, one key set at a time
  __shared__ float red_ml[NW][4][G];      // per-warp m_d, l_d, m_s, l_s

  const int c = dec_chunk_of_block(p, blockIdx.x);
  const int bg = blockIdx.y;
  const int b = bg / p.Hkv, g = bg - (bg / p.Hkv) * p.Hkv;
  const int k0 = c * DEC_CHUNK;
  const int k1 = min(k0 + DEC_CHUNK, p.n_keys);
  const int nk = k1 - k0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane % SUB, grp = lane / SUB;
  const bool chunk_has_sparse = p.all_sparse || k0 < p.sink || k1 > p.n_keys - p.window;

  float qr[G][16];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const __nv_bfloat16* qp = p.q + (long long)b * p.q_sb + (long long)(g * G + h) * p.q_sh + sub * 16;
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(qp), qr[h]);
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(qp + 8), qr[h] + 8);
#pragma unroll
    for (int e = 0; e < 16; ++e) qr[h][e] *= p.scale_log2;
  }
  float md[G], ld[G], od[G][DPL], ms[G], ls[G], os[G][DPL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    md[h] = ms[h] = -INFINITY;
    ld[h] = ls[h] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) od[h][e] = os[h][e] = 0.f;
  }
  const __nv_bfloat16* kb = p.k + (long long)b * p.k_sb + (long long)g * p.k_sh + sub * 16;
  const __nv_bfloat16* vb = p.v + (long long)b * p.v_sb + (long long)g * p.v_sh + lane * DPL;
  const int n_steps = (nk + KPW - 1) / KPW;
  // warp-uniform trip count: every lane takes part in every shuffle
  for (int s0 = warp; s0 < n_steps; s0 += NW * DEC_U) {
    uint4 kr[DEC_U][2];
    uint32_t vr[DEC_U][KPW][DPL / 2];
#pragma unroll
    for (int u = 0; u < DEC_U; ++u) {
      const int j0 = (s0 + u * NW) * KPW;  // chunk-local first key of the step
      const int jk = j0 + grp;
      const __nv_bfloat16* kp = kb + (long long)(k0 + (jk < nk ? jk : 0)) * p.k_ss;
      kr[u][0] = *reinterpret_cast<const uint4*>(kp);
      kr[u][1] = *reinterpret_cast<const uint4*>(kp + 8);
#pragma unroll
      for (int kk = 0; kk < KPW; ++kk) {
        const int jv = j0 + kk;
        const __nv_bfloat16* vp = vb + (long long)(k0 + (jv < nk ? jv : 0)) * p.v_ss;
        if constexpr (DPL == 4) {
          const uint2 w = *reinterpret_cast<const uint2*>(vp);
          vr[u][kk][0] = w.x;
          vr[u][kk][1] = w.y;
        } else {
          vr[u][kk][0] = *reinterpret_cast<const uint32_t*>(vp);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < DEC_U; ++u) {
      const int j0 = (s0 + u * NW) * KPW;
      if (j0 >= nk) break;  // warp-uniform
      {
        float kf[16];
        bf16x8_to_f32(kr[u][0], kf);
        bf16x8_to_f32(kr[u][1], kf + 8);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) d = fmaf(qr[h][e], kf[e], d);
#pragma unroll
          for (int o = SUB / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
          if (sub == 0) wsc[warp][grp][h] = d;
        }
      }
      __syncwarp();
      float sv[KPW][G];
#pragma unroll
      for (int kk = 0; kk < KPW; ++kk)
#pragma unroll
        for (int h = 0; h < G; ++h) sv[kk][h] = wsc[warp][kk][h];
      __syncwarp();
      float vf[KPW][DPL];
#pragma unroll
      for (int kk = 0; kk < KPW; ++kk)
#pragma unroll
        for (int e = 0; e < DPL / 2; ++e) {
          vf[kk][2 * e] = __uint_as_float(vr[u][kk][e] << 16);
          vf[kk][2 * e + 1] = __uint_as_float(vr[u][kk][e] & 0xffff0000u);
        }
      bool live[KPW], spk[KPW];
#pragma unroll
      for (int kk = 0; kk < KPW; ++kk) {
        live[kk] = j0 + kk < nk;
        spk[kk] = live[kk] && chunk_has_sparse && dec_sparse_key(p, k0 + j0 + kk);
      }
      // dense set
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float mx = md[h];
#pragma unroll
        for (int kk = 0; kk < KPW; ++kk) mx = live[kk] ? fmaxf(mx, sv[kk][h]) : mx;
        const float alpha = (md[h] == -INFINITY) ? 0.f : fast_exp2(md[h] - mx);
        md[h] = mx;
        ld[h] *= alpha;
#pragma unroll
        for (int e = 0; e < DPL; ++e) od[h][e] *= alpha;
#pragma unroll
        for (int kk = 0; kk < KPW; ++kk) {
          const float pk = live[kk] ? fast_exp2(sv[kk][h] - mx) : 0.f;
          ld[h] += pk;
#pragma unroll
          for (int e = 0; e < DPL; ++e) od[h][e] = fmaf(pk, vf[kk][e], od[h][e]);
        }
      }
      // sparse set (only chunks that touch the sink or the window)
      if (chunk_has_sparse) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float mx = ms[h];
#pragma unroll
          for (int kk = 0; kk < KPW; ++kk) mx = spk[kk] ? fmaxf(mx, sv[kk][h]) : mx;
          if (mx == -INFINITY) continue;
          const float alpha = (ms[h] == -INFINITY) ? 0.f : fast_exp2(ms[h] - mx);
          ms[h] = mx;
          ls[h] *= alpha;
#pragma unroll
          for (int e = 0; e < DPL; ++e) os[h][e] *= alpha;
#pragma unroll
          for (int kk = 0; kk < KPW; ++kk) {
            const float pk = spk[kk] ? fast_exp2(sv[kk][h] - mx) : 0.f;
            ls[h] += pk;
#pragma unroll
            for (int e = 0; e < DPL; ++e) os[h][e] = fmaf(pk, vf[kk][e], os[h][e]);
          }
        }
      }
    }
  }
  // ---- merge the warps' states: m = max, l and o rescaled to it ----
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      red_ml[warp][0][h] = md[h];
      red_ml[warp][1][h] = ld[h];
      red_ml[warp][2][h] = ms[h];
      red_ml[warp][3][h] = ls[h];
    }
  }
  __syncthreads();
  float* part0 = p.partials + ((long long)(b * p.H + g * G) * p.n_chunks + c) * (4 + 2 * HD);
  const long long hstride = (long long)p.n_chunks * (4 + 2 * HD);
  for (int which = 0; which < 2; ++which) {
    if (which == 1 && !chunk_has_sparse) break;  // its sparse m stays -inf: the merge skips it
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) M = fmaxf(M, red_ml[w][2 * which][h]);
      const float mine = red_ml[warp][2 * which][h];
      const float sc = (mine == -INFINITY) ? 0.f : fast_exp2(mine - M);
#pragma unroll
      for (int e = 0; e < DPL; ++e) red_o[warp][h][lane * DPL + e] = (which == 0 ? od[h][e] : os[h][e]) * sc;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * HD; idx += DEC_THREADS) {
      const int h = idx / HD, t = idx - (idx / HD) * HD;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) sum += red_o[w][h][t];
      float* part = part0 + h * hstride;
      part[4 + which * HD + t] = sum;
      if (t == 0) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, red_ml[w][2 * which][h]);
        float L = 0.f;
        if (M != -INFINITY) {
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const float m = red_ml[w][2 * which][h];
            if (m != -INFINITY) L += red_ml[w][2 * which + 1][h] * fast_exp2(m - M);
          }
        }
        part[2 * which] = M;
        part[2 * which + 1] = L;
        if (which == 0 && !chunk_has_sparse) {
          part[2] = -INFINITY;
          part[3] = 0.f;
        }
      }
    }
    __syncthreads();
  }
}

// Merge partials of every chunk that was launched: grid (B*H), block HD.
// Chunk statistics are read in batches of 8 independent loads.
template <int HD>
__global__ void decode_merge_kernel(const __grid_constant__ DecodeParams p) {
  const int bh = blockIdx.x;
  const int t = threadIdx.x;
  const float* base = p.partials + (long long)bh * p.n_chunks * (4 + 2 * HD);
  for (int which = 0; which < 2; ++which) {
    __nv_bfloat16* dst = which == 0 ? p.dense_out : p.sparse_out;
    if (!dst) continue;
    const int mo = which == 0 ? 0 : 2;
    float M = -INFINITY;
    for (int x0 = 0; x0 < p.n_launched; x0 += 8) {
      float mv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int x = x0 + u;
        mv[u] = x < p.n_launched ? base[(long long)dec_chunk_of_block(p, x) * (4 + 2 * HD) + mo] : -INFINITY;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) M = fmaxf(M, mv[u]);
    }
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int x0 = 0; x0 < p.n_launched; x0 += 8) {
        float mv[8], lv[8], ov[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int x = x0 + u;
          if (x < p.n_launched) {
            const float* part = base + (long long)dec_chunk_of_block(p, x) * (4 + 2 * HD);
            mv[u] = part[mo];
            lv[u] = part[mo + 1];
            ov[u] = part[4 + which * HD + t];
          } else {
            mv[u] = -INFINITY;
            lv[u] = ov[u] = 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (mv[u] == -INFINITY) continue;
          const float w = fast_exp2(mv[u] - M);
          L += lv[u] * w;
          O += ov[u] * w;
        }
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    dst[((long long)b * p.H + h) * HD + t] = __float2bfloat16_rn(o);
  }
}

template <int HD, int G>
static void launch_partial(const DecodeParams& p, dim3 grid, cudaStream_t stream) {
  decode_partial_kernel<HD, G><<<grid, DEC_THREADS, 0, stream>>>(p);
}

template <int HD>
static void launch_hd(const DecodeParams& p, dim3 grid, cudaStream_t stream) {
  switch (p.G) {
    case 1: launch_partial<HD, 1>(p, grid, stream); break;
    case 2: launch_partial<HD, 2>(p, grid, stream); break;
    case 3: launch_partial<HD, 3>(p, grid, stream); break;
    case 4: launch_partial<HD, 4>(p, grid, stream); break;
    case 5: launch_partial<HD, 5>(p, grid, stream); break;
    case 6: launch_partial<HD, 6>(p, grid, stream); break;
    case 7: launch_partial<HD, 7>(p, grid, stream); break;
    default: launch_partial<HD, 8>(p, grid, stream); break;
  }
  decode_merge_kernel<HD><<<p.B * p.H, HD, 0, stream>>>(p);
}

cudaError_t launch_decode(const DecodeParams& p, int head_dim, cudaStream_t stream) {
  dim3 grid(p.n_launched, p.B * p.Hkv);
  if (head_dim == 128) launch_hd<128>(p, grid, stream);
  else launch_hd<64>(p, grid, stream);
  return cudaGetLastError();
}

}  // namespace dta
