// Internal launch parameters of the decode kernels (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace dta {

// Keys per split-K chunk.  The dense set uses the longest chunk up to
// DEC_DENSE_CHUNK_MAX that still gives every SM a CTA (long streams per CTA,
// few partials), never below DEC_DENSE_CHUNK_MIN; the sparse set uses the
// shortest chunk whose sink and window chunks fit one thread-block cluster
// (at most DEC_SPARSE_CLUSTER_CHUNK_MAX keys), else DEC_SPARSE_CHUNK.  All are
// multiples of the 64-key shared-memory stage.
#ifndef DTA_DEC_DENSE_CHUNK
#define DTA_DEC_DENSE_CHUNK 4096
#endif
#ifndef DTA_DEC_SPARSE_CHUNK
#define DTA_DEC_SPARSE_CHUNK 256
#endif
constexpr int DEC_DENSE_CHUNK_MAX = DTA_DEC_DENSE_CHUNK;
constexpr int DEC_DENSE_CHUNK_MIN = 256;
constexpr int DEC_SPARSE_CHUNK = DTA_DEC_SPARSE_CHUNK;
#ifndef DTA_DEC_SPARSE_CLUSTER_CHUNK_MAX
#define DTA_DEC_SPARSE_CLUSTER_CHUNK_MAX 512
#endif
constexpr int DEC_SPARSE_CLUSTER_CHUNK_MAX = DTA_DEC_SPARSE_CLUSTER_CHUNK_MAX;
// Largest thread-block cluster for the in-cluster merge of the sparse set
// (sizes above 8 are the non-portable ones, checked against the device by
// an occupancy query before use).
constexpr int DEC_CLUSTER_MAX = 16;
// Cluster size the sparse chunking aims for (at most DEC_CLUSTER_MAX): the
// shortest chunk whose sink and window chunks number at most this many.  At
// config-2 shapes (sink 128, window 2048) 9 gives 256-key chunks: 8.45 us per
// sparse step against 8.7 us at 16 (192-key chunks) and 10.5 us at 5
// (512-key chunks), same box.
#ifndef DTA_DEC_CLUSTER_TARGET
#define DTA_DEC_CLUSTER_TARGET 9
#endif
constexpr int DEC_CLUSTER_TARGET = DTA_DEC_CLUSTER_TARGET;
static_assert(DEC_CLUSTER_TARGET >= 1 && DEC_CLUSTER_TARGET <= DEC_CLUSTER_MAX, "cluster target");

// Chunking of one key set.  The sparse set's chunking depends on (sink,
// window) only, so a sparse row is bit-identical whether it comes from an
// anchor step (dense + sparse) or from a non-anchor step (sparse only).  Its
// chunks tile [0, sink) and then [n - window, n) from that range's first key
// (with n <= sink + window: [0, n), like the dense set).
struct DecodeSet {
  int chunk;               // keys per chunk
  int n_chunks;            // chunks covering the cache
  int n_launched;          // chunks launched (all, or the sink + window chunks)
  int n_sink_chunks;       // sparse set: chunks covering [0, sink)
  int sparse;              // 1: the sink + window layout
  float* partials;         // [B, H, n_launched, 4 + d]: (m, l, -, -, o[d]) per launched chunk
};

struct DecodeParams {
  const __nv_bfloat16* q;
  long long q_sb, q_sh;
  const __nv_bfloat16* k;
  long long k_sb, k_sh, k_ss;
  const __nv_bfloat16* v;
  long long v_sb, v_sh, v_ss;
  int B, H, Hkv, G, n_keys;
  // optional device key count (CUDA-graph replays with a growing cache): the
  // kernels read the live count n = clamp(*n_keys_dev, 1, n_keys) and n_keys
  // is the capacity the grids are sized for; all_sparse is then decided per
  // call on the device (n <= sink + window)
  const int* n_keys_dev;
  float scale_log2;
  int window, sink, all_sparse;
  DecodeSet set[2];        // 0: dense (every key), 1: sparse
  __nv_bfloat16* dense_out;
  __nv_bfloat16* sparse_out;
  int sparse_merged;       // set by the launcher: the sparse set merged in-cluster
};

cudaError_t launch_decode(const DecodeParams& p, int head_dim, cudaStream_t stream);

}  // namespace dta
