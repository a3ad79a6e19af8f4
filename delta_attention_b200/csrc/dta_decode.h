// Internal launch parameters of the decode kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace dta {

constexpr int DEC_CHUNK = 512;  // keys per split-K chunk

struct DecodeParams {
  const __nv_bfloat16* q;
  long long q_sb, q_sh;
  const __nv_bfloat16* k;
  long long k_sb, k_sh, k_ss;
  const __nv_bfloat16* v;
  long long v_sb, v_sh, v_ss;
  int B, H, Hkv, G, n_keys;
  float scale_log2;
  int window, sink, all_sparse;
  int want_dense;
  int n_chunks;            // chunks covering the cache
  int n_launched;          // chunks launched (all, or the sparse-set chunks)
  int n_sink_chunks;       // chunks covering [0, sink)
  int first_window_chunk;  // first chunk touching [n_keys - window, n_keys)
  float* partials;         // [B, H, n_chunks, 4 + 2 * d]
  __nv_bfloat16* dense_out;
  __nv_bfloat16* sparse_out;
};

cudaError_t launch_decode(const DecodeParams& p, int head_dim, cudaStream_t stream);

}  // namespace dta
