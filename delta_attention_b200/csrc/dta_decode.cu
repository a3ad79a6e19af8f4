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
constexpr int DEC_GMAX = 8;  // max query heads per KV head

__device__ __forceinline__ bool dec_sparse_key(const DecodeParams& p, int j) {
  return p.all_sparse || j < p.sink || j >= p.n_keys - p.window;
}

__device__ __forceinline__ int dec_chunk_of_block(const DecodeParams& p, int x) {
  if (p.want_dense || p.all_sparse) return x;
  return x < p.n_sink_chunks ? x : p.first_window_chunk + (x - p.n_sink_chunks);
}

template <int HD>
__global__ void __launch_bounds__(DEC_THREADS) decode_partial_kernel(const __grid_constant__ DecodeParams p) {
  constexpr int SUB = HD / 16;  // lanes per key in the QK pass (16 dims each)
  constexpr int KPW = 32 / SUB; // keys per warp step
  __shared__ float sc[DEC_GMAX][DEC_CHUNK];
  __shared__ float red[4][DEC_GMAX][HD];
  __shared__ float stat[4][DEC_GMAX];  // m_d, l_d, m_s, l_s

  const int c = dec_chunk_of_block(p, blockIdx.x);
  const int bg = blockIdx.y;
  const int b = bg / p.Hkv, g = bg - (bg / p.Hkv) * p.Hkv;
  const int G = p.G;
  const int k0 = c * DEC_CHUNK;
  const int k1 = min(k0 + DEC_CHUNK, p.n_keys);
  const int nk = k1 - k0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool chunk_has_sparse = p.all_sparse || k0 < p.sink || k1 > p.n_keys - p.window;

  // ---- pass 1: scores (log2 domain) ----
  {
    const int sub = lane % SUB, grp = lane / SUB;
    float qr[DEC_GMAX][16];
#pragma unroll
    for (int h = 0; h < DEC_GMAX; ++h) {
      if (h < G) {
        const __nv_bfloat16* qp = p.q + (long long)b * p.q_sb + (long long)(g * G + h) * p.q_sh + sub * 16;
        const uint4 u0 = *reinterpret_cast<const uint4*>(qp);
        const uint4 u1 = *reinterpret_cast<const uint4*>(qp + 8);
        const __nv_bfloat162* v0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
        const __nv_bfloat162* v1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f0 = __bfloat1622float2(v0[e]);
          const float2 f1 = __bfloat1622float2(v1[e]);
          qr[h][2 * e] = f0.x * p.scale_log2;
          qr[h][2 * e + 1] = f0.y * p.scale_log2;
          qr[h][8 + 2 * e] = f1.x * p.scale_log2;
          qr[h][8 + 2 * e + 1] = f1.y * p.scale_log2;
        }
      }
    }
    const __nv_bfloat16* kb = p.k + (long long)b * p.k_sb + (long long)g * p.k_sh + sub * 16;
    // warp-uniform trip count: every lane takes part in every shuffle
    for (int base = warp * KPW; base < nk; base += 4 * KPW) {
      const int jj = base + grp;
      const bool valid = jj < nk;
      float kf[16];
      if (valid) {
        const __nv_bfloat16* kp = kb + (long long)(k0 + jj) * p.k_ss;
        const uint4 u0 = *reinterpret_cast<const uint4*>(kp);
        const uint4 u1 = *reinterpret_cast<const uint4*>(kp + 8);
        const __nv_bfloat162* v0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
        const __nv_bfloat162* v1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f0 = __bfloat1622float2(v0[e]);
          const float2 f1 = __bfloat1622float2(v1[e]);
          kf[2 * e] = f0.x; kf[2 * e + 1] = f0.y; kf[8 + 2 * e] = f1.x; kf[8 + 2 * e + 1] = f1.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) kf[e] = 0.f;
      }
#pragma unroll
      for (int h = 0; h < DEC_GMAX; ++h) {
        if (h < G) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) d = fmaf(qr[h][e], kf[e], d);
#pragma unroll
          for (int o = SUB / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
          if (valid && sub == 0) sc[h][jj] = d;
        }
      }
    }
  }
  __syncthreads();

  // ---- pass 2: per-head max / sum over the chunk (dense and sparse sets) ----
  for (int h = warp; h < G; h += 4) {
    float md = -INFINITY, ms = -INFINITY;
    for (int jj = lane; jj < nk; jj += 32) {
      const float s = sc[h][jj];
      md = fmaxf(md, s);
      if (dec_sparse_key(p, k0 + jj)) ms = fmaxf(ms, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      md = fmaxf(md, __shfl_xor_sync(0xffffffffu, md, o));
      ms = fmaxf(ms, __shfl_xor_sync(0xffffffffu, ms, o));
    }
    float ld = 0.f, ls = 0.f;
    for (int jj = lane; jj < nk; jj += 32) {
      const float s = sc[h][jj];
      const float pd = fast_exp2(s - md);
      ld += pd;
      if (ms != -INFINITY && dec_sparse_key(p, k0 + jj)) ls += fast_exp2(s - ms);
      sc[h][jj] = pd;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ld += __shfl_xor_sync(0xffffffffu, ld, o);
      ls += __shfl_xor_sync(0xffffffffu, ls, o);
    }
    if (lane == 0) {
      stat[0][h] = md;
      stat[1][h] = ld;
      stat[2][h] = ms;
      stat[3][h] = ls;
    }
  }
  __syncthreads();

  // ---- pass 3: P.V (lane owns HD/32 dims; warps split keys) ----
  {
    constexpr int DPL = HD / 32;
    float od[DEC_GMAX][DPL], os[DEC_GMAX][DPL];
    float sr[DEC_GMAX];
#pragma unroll
    for (int h = 0; h < DEC_GMAX; ++h) {
      sr[h] = (h < G && stat[2][h] != -INFINITY) ? fast_exp2(stat[0][h] - stat[2][h]) : 0.f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) od[h][e] = os[h][e] = 0.f;
    }
    const __nv_bfloat16* vb = p.v + (long long)b * p.v_sb + (long long)g * p.v_sh + lane * DPL;
    for (int jj = warp; jj < nk; jj += 4) {
      const __nv_bfloat16* vp = vb + (long long)(k0 + jj) * p.v_ss;
      float vf[DPL];
      if constexpr (DPL == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(vp);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 c2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        vf[0] = a.x; vf[1] = a.y; vf[2] = c2.x; vf[3] = c2.y;
      } else {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vp));
        vf[0] = a.x; vf[1] = a.y;
      }
      const bool sp = chunk_has_sparse && dec_sparse_key(p, k0 + jj);
#pragma unroll
      for (int h = 0; h < DEC_GMAX; ++h) {
        if (h < G) {
          const float pd = sc[h][jj];
#pragma unroll
          for (int e = 0; e < DPL; ++e) od[h][e] = fmaf(pd, vf[e], od[h][e]);
          if (sp) {
#pragma unroll
            for (int e = 0; e < DPL; ++e) os[h][e] = fmaf(pd, vf[e], os[h][e]);
          }
        }
      }
    }
    // cross-warp reduction, dense set then sparse set, through one buffer
    float* part0 = p.partials + ((long long)(b * p.H + g * G) * p.n_chunks + c) * (4 + 2 * HD);
    const long long hstride = (long long)p.n_chunks * (4 + 2 * HD);
    for (int which = 0; which < 2; ++which) {
#pragma unroll
      for (int h = 0; h < DEC_GMAX; ++h) {
        if (h < G) {
#pragma unroll
          for (int e = 0; e < DPL; ++e)
            red[warp][h][lane * DPL + e] = which == 0 ? od[h][e] : os[h][e] * sr[h];
        }
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < G * HD; idx += DEC_THREADS) {
        const int h = idx / HD, t = idx - (idx / HD) * HD;
        const float sum = red[0][h][t] + red[1][h][t] + red[2][h][t] + red[3][h][t];
        float* part = part0 + h * hstride;
        part[4 + which * HD + t] = sum;
        if (which == 0 && t < 4) part[t] = stat[t][h];
      }
      __syncthreads();
    }
  }
}

// Merge partials of every chunk that was launched: grid (B*H), block HD.
template <int HD>
__global__ void decode_merge_kernel(const __grid_constant__ DecodeParams p) {
  const int bh = blockIdx.x;
  const int t = threadIdx.x;
  const float* base = p.partials + (long long)bh * p.n_chunks * (4 + 2 * HD);
  for (int which = 0; which < 2; ++which) {
    __nv_bfloat16* dst = which == 0 ? p.dense_out : p.sparse_out;
    if (!dst) continue;
    float M = -INFINITY;
    for (int x = 0; x < p.n_launched; ++x) {
      const int c = dec_chunk_of_block(p, x);
      M = fmaxf(M, base[(long long)c * (4 + 2 * HD) + (which == 0 ? 0 : 2)]);
    }
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int x = 0; x < p.n_launched; ++x) {
        const int c = dec_chunk_of_block(p, x);
        const float* part = base + (long long)c * (4 + 2 * HD);
        const float m = part[which == 0 ? 0 : 2];
        if (m == -INFINITY) continue;
        const float w = fast_exp2(m - M);
        L += part[which == 0 ? 1 : 3] * w;
        O += part[4 + which * HD + t] * w;
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    dst[((long long)b * p.H + h) * HD + t] = __float2bfloat16_rn(o);
  }
}

cudaError_t launch_decode(const DecodeParams& p, int head_dim, cudaStream_t stream) {
  dim3 grid(p.n_launched, p.B * p.Hkv);
  if (head_dim == 128) {
    decode_partial_kernel<128><<<grid, DEC_THREADS, 0, stream>>>(p);
    decode_merge_kernel<128><<<p.B * p.H, 128, 0, stream>>>(p);
  } else {
    decode_partial_kernel<64><<<grid, DEC_THREADS, 0, stream>>>(p);
    decode_merge_kernel<64><<<p.B * p.H, 64, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace dta
