// extern "C" entry points of libdelta_attention_b200.so: argument validation,
// workspace layout, TMA tensor-map encoding and kernel launches.  No entry
// point allocates device memory; all scratch comes from the caller's workspace.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "delta_attention_b200.h"
#include "dta_decode.h"
#include "dta_internal.h"
#include "dta_prefill.h"
#include "dta_ptx.cuh"

namespace {
thread_local int g_last_cuda_error = 0;
}  // namespace

namespace dta {

int fail_cuda(cudaError_t e) {
  g_last_cuda_error = (int)e;
  (void)cudaGetLastError();  // clear the runtime's pending (non-sticky) error
  return DTA_ERR_CUDA;
}

int check_device(int* sms) {
  struct DeviceInfo {
    int ok = -1;
    int sms = 0;
  };
  static DeviceInfo info[64];
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e);
  if (dev < 0 || dev >= 64) return DTA_ERR_UNSUPPORTED_DEVICE;
  // Make the device's primary context current on this thread: the TMA
  // descriptor encode is a driver call that needs a current context, which a
  // host thread that has made no context-creating runtime call yet (a fresh
  // worker thread) does not have.
  if ((e = cudaSetDevice(dev)) != cudaSuccess) return fail_cuda(e);
  std::lock_guard<std::mutex> lock(mu);
  if (info[dev].ok < 0) {
    int major = 0, n = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return fail_cuda(e);
    if ((e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return fail_cuda(e);
    info[dev].ok = (major == 10) ? 1 : 0;
    info[dev].sms = n;
  }
  if (!info[dev].ok) return DTA_ERR_UNSUPPORTED_DEVICE;
  *sms = info[dev].sms;
  return DTA_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 4-D bf16 tensor map over (d, rows, heads, batch) with a 128-byte swizzle.
int encode_4d(CUtensorMap* map, const void* base, int d, long long rows, int heads, int batch, long long s_row,
              long long s_head, long long s_batch, int box_rows, int box_heads) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) {
    g_last_cuda_error = (int)CUDA_ERROR_NOT_FOUND;
    return DTA_ERR_CUDA;
  }
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(s_row * 2), (cuuint64_t)(s_head * 2), (cuuint64_t)(s_batch * 2)};
  cuuint32_t box[4] = {64u, (cuuint32_t)box_rows, (cuuint32_t)box_heads, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) return DTA_OK;
  g_last_cuda_error = (int)r;  // the driver's CUresult, reported by dta_last_cuda_error
  return DTA_ERR_CUDA;
}

}  // namespace dta

namespace {

constexpr size_t kHeaderBytes = 256;  // job counter, error word

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

using dta::check_device;
using dta::fail_cuda;

using dta::encode_4d;

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
inline bool stride_ok(long long s) { return s > 0 && (s * 2) % 16 == 0; }

// ---------------------------------------------------------------------------
// split-K plan of the rows launch's dense jobs
// ---------------------------------------------------------------------------
// The dense row tiles are cut into chunks of at most (total key tiles) /
// (SMs * kSplitFactor) key tiles, so the longest row tile (the dense tail,
// every key) no longer bounds the launch and the longest-first schedule
// balances; chunks are never shorter than kSplitMinTiles (unless the caller
// forces a chunk length).
#ifndef DTA_SPLIT_FACTOR
#define DTA_SPLIT_FACTOR 3
#endif
#ifndef DTA_SPLIT_MIN_TILES
#define DTA_SPLIT_MIN_TILES 16
#endif
constexpr int kSplitFactor = DTA_SPLIT_FACTOR;
constexpr int kSplitMinTiles = DTA_SPLIT_MIN_TILES;
constexpr int kMaxChunks = 16384;  // chunks per row tile (the kernel packs the count in 15 bits)

struct RowsSplit {
  int n_dense_tiles = 0;
  int c = 0, cmax = 1;     // PrefillParams::split_c / split_cmax
  size_t cnt_bytes = 0;    // part_cnt, zeroed with the header
  size_t part_o_bytes = 0, part_lse_bytes = 0;
};

// `tiles_of(t)` = key tiles of row tile t's longest row (estimated when the
// rows come from a device list); `extra` = key tiles of the other jobs;
// `forced` > 0 fixes the chunk length.
template <class F>
RowsSplit plan_rows_split(int BG, int n_sel, int JR, int head_dim, int sms, long long extra, int forced, F tiles_of) {
  RowsSplit S;
  S.n_dense_tiles = (n_sel + JR - 1) / JR;
  long long total = extra;
  int t_max = 1;
  for (int t = 0; t < S.n_dense_tiles; ++t) {
    const int T = tiles_of(t);
    total += (long long)T * BG;
    if (T > t_max) t_max = T;
  }
  const long long c0 = (total + (long long)sms * kSplitFactor - 1) / ((long long)sms * kSplitFactor);
  // no split when the longest row tile is within 10% of the work per SM: the
  // longest-first order of whole tiles is then balanced already
  if (forced <= 0 && (long long)t_max * 10 <= total * 11 / sms) return S;
  int chunk = forced > 0 ? forced : (int)(c0 < kSplitMinTiles ? kSplitMinTiles : c0);
  if ((t_max + chunk - 1) / chunk > kMaxChunks) chunk = (t_max + kMaxChunks - 1) / kMaxChunks;
  const int cmax = (t_max + chunk - 1) / chunk;
  if (cmax <= 1) return S;
  S.cmax = cmax;
  S.c = chunk;
  const size_t slots = (size_t)BG * S.n_dense_tiles * cmax * dta::PREFILL_NQ * 128;
  S.part_o_bytes = align_up(slots * head_dim * 4, 256);
  S.part_lse_bytes = align_up(slots * 4, 256);
  S.cnt_bytes = align_up((size_t)BG * S.n_dense_tiles * dta::PREFILL_NQ * 4 * 4, 256);  // per warp
  return S;
}

// SM count of the current device for sizing (148, a B200's, when there is none)
int sizing_sms() {
  int sms = 0;
  if (check_device(&sms) != DTA_OK || sms <= 0) sms = 148;
  return sms;
}

// ---------------------------------------------------------------------------
// prefill layout
// ---------------------------------------------------------------------------
// workspace: header (job counter, error word) | split counters | dense_buf |
// sparse_buf | delta_buf | split partials (O, lse)
struct PrefillLayout {
  int s_p, n_anchor, n_sel;
  bool fuse;           // the windowed launch forms delta itself (no sparse anchor jobs)
  bool delta_cross;    // ... in the first job of each anchor period, for the period's other tiles
  int win_group;       // windowed jobs per anchor period when it spans several, else 1
  int n_sparse_tiles;  // sparse anchor row tiles of the rows launch
  RowsSplit split;
  size_t buf_bytes;    // one of dense_buf / sparse_buf (fp32)
  size_t delta_bytes;  // delta_buf (bf16)
  size_t ws_bytes;
};

int prefill_layout(const dta_prefill_args* a, int sms, PrefillLayout* L) {
  if (!a) return DTA_ERR_INVALID_ARG;
  if (a->abi_version != DTA_ABI_VERSION) return DTA_ERR_INVALID_ARG;
  if (a->batch <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->seq_len <= 0) return DTA_ERR_SHAPE;
  if (a->head_dim != 64 && a->head_dim != 128) return DTA_ERR_HEAD_DIM;
  if (a->n_heads % a->n_kv_heads != 0) return DTA_ERR_SHAPE;
  const int G = a->n_heads / a->n_kv_heads;
  if (G > 128 || 128 % G != 0) return DTA_ERR_SHAPE;
  if (a->mode < 0 || a->mode > 2) return DTA_ERR_INVALID_ARG;
  if (a->window < 0 || a->sink < 0 || a->q_block <= 0 || a->split_tiles < 0) return DTA_ERR_INVALID_ARG;
  const int s = a->seq_len;
  if (a->mode == DTA_MODE_SPARSE_ONLY) {
    L->s_p = s;
    L->n_anchor = 0;
    L->n_sel = 0;
  } else if (a->anchors) {
    if (a->n_anchors <= 0 || a->s_p <= 0 || a->s_p > s || a->n_anchors > a->s_p) return DTA_ERR_INVALID_ARG;
    L->s_p = a->s_p;
    L->n_anchor = a->n_anchors;
    // with the anchors' deltas given, the rows launch computes the tail only
    L->n_sel = (a->anchor_delta_in ? 0 : a->n_anchors) + (s - a->s_p);
  } else {
    if (a->anchor_delta_in) return DTA_ERR_INVALID_ARG;  // only with explicit anchors
    if (a->gamma <= 0) return DTA_ERR_GAMMA;
    const int cut_n = s % a->gamma + (a->gamma > 128 ? a->gamma : 128);
    const int s_p = s - cut_n;
    if (s_p < 0 || s_p % a->gamma != 0) return DTA_ERR_GAMMA;
    L->s_p = s_p;
    L->n_anchor = s_p / a->gamma;
    L->n_sel = L->n_anchor + cut_n;
  }
  // With uniform anchors, 4 or 8 heads per KV group and gamma a power of two
  // >= 8, the windowed launch forms delta = dense - sparse itself from each
  // anchor row's own sparse output, and the rows launch skips the sparse anchor
  // rows (and the delta kernel).  Both phases derive the choice from the
  // arguments alone.
  const int R = 128 / G, JR = dta::PREFILL_NQ * R, BG = a->batch * a->n_kv_heads;
  const bool pow2 = a->gamma >= 8 && (a->gamma & (a->gamma - 1)) == 0;
  L->fuse = a->mode == DTA_MODE_DELTA && !a->anchors && L->n_anchor > 0 && (G == 4 || G == 8) && pow2;
  L->delta_cross = L->fuse && a->gamma > R;
  L->win_group = (L->fuse && a->gamma > JR) ? a->gamma / JR : 1;
  const bool have_delta = a->anchor_delta_in != nullptr;
  if (have_delta && (a->mode != DTA_MODE_DELTA || a->anchor_delta)) return DTA_ERR_INVALID_ARG;
  L->n_sparse_tiles = (a->mode == DTA_MODE_DELTA && !L->fuse && !have_delta) ? (L->n_anchor + JR - 1) / JR : 0;
  if (L->n_sel > 0) {
    // a sparse anchor tile spans its rows' window plus the rows' own spread
    const long long sparse_tiles =
        (long long)L->n_sparse_tiles * BG * ((a->window + a->sink) / dta::PREFILL_BN + 2);
    const int n_anchor = have_delta ? 0 : L->n_anchor, s_p = L->s_p, n_sel = L->n_sel, gamma = a->gamma;
    const bool uniform = !a->anchors;
    auto tiles_of = [&](int t) {
      const int i = (t + 1) * JR < n_sel ? (t + 1) * JR - 1 : n_sel - 1;  // last list row of tile t
      long long pos;
      if (i >= n_anchor) pos = s_p + (i - n_anchor);
      else if (uniform) pos = (long long)i * gamma;
      else pos = (long long)s_p * i / n_anchor;  // explicit anchors: spread estimate
      return (int)(pos / dta::PREFILL_BN) + 1;
    };
    L->split = plan_rows_split(BG, L->n_sel, JR, a->head_dim, sms, sparse_tiles, a->split_tiles, tiles_of);
  } else {
    L->split = RowsSplit();
  }
  const bool need_bufs = a->mode == DTA_MODE_DELTA && L->n_anchor > 0 && !have_delta;
  L->buf_bytes = need_bufs ? align_up((size_t)a->batch * L->n_anchor * a->n_heads * a->head_dim * 4, 256) : 0;
  L->delta_bytes = need_bufs ? align_up((size_t)a->batch * L->n_anchor * a->n_heads * a->head_dim * 2, 256) : 0;
  L->ws_bytes = kHeaderBytes + L->split.cnt_bytes + 2 * L->buf_bytes + L->delta_bytes + L->split.part_o_bytes +
                L->split.part_lse_bytes;
  return DTA_OK;
}

}  // namespace

extern "C" {

int dta_abi_version(void) { return DTA_ABI_VERSION; }

int dta_last_cuda_error(void) { return g_last_cuda_error; }

const char* dta_status_string(int st) {
  switch (st) {
    case DTA_OK: return "ok";
    case DTA_ERR_INVALID_ARG: return "invalid argument";
    case DTA_ERR_SHAPE: return "inconsistent shape";
    case DTA_ERR_STRIDE: return "unsupported stride (head_dim must be contiguous, strides multiples of 16 bytes)";
    case DTA_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case DTA_ERR_GAMMA: return "gamma incompatible with seq_len (s_p % gamma != 0 or seq_len < cut_n)";
    case DTA_ERR_HEAD_DIM: return "head_dim not supported (64 or 128)";
    case DTA_ERR_WORKSPACE: return "workspace missing or too small";
    case DTA_ERR_CUDA: return "CUDA runtime error";
    case DTA_ERR_UNSUPPORTED_DEVICE: return "device is not sm_100 (B200)";
    case DTA_ERR_KERNEL_TIMEOUT: return "kernel gave up on a bounded wait";
    case DTA_ERR_SCRATCH_LIMIT: return "request needs more scratch than the no-alloc entry point's static array";
    default: return "unknown status";
  }
}

size_t dta_prefill_workspace_size(const dta_prefill_args* a) {
  PrefillLayout L;
  if (prefill_layout(a, sizing_sms(), &L) != DTA_OK) return 0;
  return L.ws_bytes;
}

int dta_prefill(const dta_prefill_args* a, void* stream_) {
  PrefillLayout L;
  int st = prefill_layout(a, 148, &L);  // argument checks (sized again below for this device)
  if (st != DTA_OK) return st;
  if (!a->workspace) return DTA_ERR_WORKSPACE;
  if (!a->q || !a->k || !a->v || !a->out) return DTA_ERR_INVALID_ARG;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out)) return DTA_ERR_ALIGNMENT;
  if (!stride_ok(a->q_stride_s) || !stride_ok(a->q_stride_h) || !stride_ok(a->q_stride_b) ||
      !stride_ok(a->k_stride_s) || !stride_ok(a->k_stride_h) || !stride_ok(a->k_stride_b) ||
      !stride_ok(a->v_stride_s) || !stride_ok(a->v_stride_h) || !stride_ok(a->v_stride_b))
    return DTA_ERR_STRIDE;
  if (a->anchor_delta && (a->mode != DTA_MODE_DELTA || !aligned16(a->anchor_delta))) return DTA_ERR_INVALID_ARG;
  if (a->anchor_delta_in && !aligned16(a->anchor_delta_in)) return DTA_ERR_ALIGNMENT;
  if (a->phases < 0 || a->phases > (DTA_PHASE_ROWS | DTA_PHASE_WINDOW)) return DTA_ERR_INVALID_ARG;
  if (a->wait_cycles < 0 || (a->flags & ~DTA_FLAG_TEST_STALL) != 0) return DTA_ERR_INVALID_ARG;
  if (a->error_word && ((uintptr_t)a->error_word & 3u) != 0) return DTA_ERR_ALIGNMENT;
  if ((a->lse_sparse && ((uintptr_t)a->lse_sparse & 3u) != 0) || (a->lse_dense && ((uintptr_t)a->lse_dense & 3u) != 0))
    return DTA_ERR_ALIGNMENT;
  // the dense rows' log-sum-exp is indexed by the full list (anchors, tail)
  if (a->lse_dense && a->anchor_delta_in) return DTA_ERR_INVALID_ARG;
  const int phases = a->phases ? a->phases : (DTA_PHASE_ROWS | DTA_PHASE_WINDOW);
  int sms = 0;
  if ((st = check_device(&sms)) != DTA_OK) return st;
  if ((st = prefill_layout(a, sms, &L)) != DTA_OK) return st;
  if (a->workspace_bytes < L.ws_bytes || !aligned16(a->workspace)) return DTA_ERR_WORKSPACE;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);

  dta::PrefillParams p;
  memset(&p, 0, sizeof(p));
  const int B = a->batch, H = a->n_heads, Hkv = a->n_kv_heads, S = a->seq_len, d = a->head_dim;
  const int G = H / Hkv, R = 128 / G, JR = dta::PREFILL_NQ * R;
  p.q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  p.q_sb = a->q_stride_b; p.q_sh = a->q_stride_h; p.q_ss = a->q_stride_s;
  p.B = B; p.H = H; p.Hkv = Hkv; p.G = G; p.R = R;
  p.scale_log2 = a->scaling * 1.4426950408889634f;
  p.window = a->window; p.sink = a->sink; p.qblock = a->q_block;
  p.gamma = a->gamma; p.s_p = L.s_p; p.n_anchor = L.n_anchor; p.n_sel = L.n_sel;
  dta::fast_div_params(p.qblock, &p.qblock_mul, &p.qblock_sh);
  if (p.gamma > 0) dta::fast_div_params(p.gamma, &p.gamma_mul, &p.gamma_sh);
  p.anchors = a->anchors;
  p.mode = a->mode;
  p.out_rows = S;
  p.seq_q = S;
  p.kv_len = S;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.wait_cycles = a->wait_cycles > 0 ? a->wait_cycles : dta::kWaitTimeoutCycles;
  p.test_stall = (a->flags & DTA_FLAG_TEST_STALL) ? 1 : 0;
  p.lse_sparse = a->lse_sparse;
  p.lse_dense = a->lse_dense;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  p.counter = reinterpret_cast<int*>(ws);
  p.error = a->error_word ? a->error_word : reinterpret_cast<int*>(ws) + 1;
  uint8_t* cur = ws + kHeaderBytes;
  p.part_cnt = L.split.cnt_bytes ? reinterpret_cast<int*>(cur) : nullptr;
  cur += L.split.cnt_bytes;
  p.dense_buf = L.buf_bytes ? reinterpret_cast<float*>(cur) : nullptr;
  p.sparse_buf = L.buf_bytes ? reinterpret_cast<float*>(cur + L.buf_bytes) : nullptr;
  cur += 2 * L.buf_bytes;
  __nv_bfloat16* delta_buf = L.delta_bytes ? reinterpret_cast<__nv_bfloat16*>(cur) : nullptr;
  // given deltas (explicit anchors) replace the delta kernel's output
  p.delta_buf = a->anchor_delta_in ? reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(a->anchor_delta_in)) : delta_buf;
  cur += L.delta_bytes;
  p.part_o = L.split.part_o_bytes ? reinterpret_cast<float*>(cur) : nullptr;
  cur += L.split.part_o_bytes;
  p.part_lse = L.split.part_lse_bytes ? reinterpret_cast<float*>(cur) : nullptr;

  if ((st = encode_4d(&p.tm_k, a->k, d, S, Hkv, B, a->k_stride_s, a->k_stride_h, a->k_stride_b, dta::PREFILL_BN, 1)) != DTA_OK)
    return st;
  if ((st = encode_4d(&p.tm_v, a->v, d, S, Hkv, B, a->v_stride_s, a->v_stride_h, a->v_stride_b, dta::PREFILL_BN, 1)) != DTA_OK)
    return st;
  if ((st = encode_4d(&p.tm_q, a->q, d, S, H, B, a->q_stride_s, a->q_stride_h, a->q_stride_b, R, G)) != DTA_OK)
    return st;

  // the job counter, the workspace error word and the split counters start
  // at zero (the ROWS phase uses them; a WINDOW-only call keeps the error word
  // of the ROWS call before it)
  cudaError_t e;
  if (phases & DTA_PHASE_ROWS) {
    e = cudaMemsetAsync(a->workspace, 0, kHeaderBytes + L.split.cnt_bytes, stream);
    if (e != cudaSuccess) return fail_cuda(e);
  }
  const bool fuse = L.fuse;
  bool rows_launched = false;
  // launch 1: dense rows (anchors + tail) and, unless fused, sparse anchor rows
  if ((phases & DTA_PHASE_ROWS) && a->mode != DTA_MODE_SPARSE_ONLY && L.n_sel > 0) {
    dta::PrefillParams r = p;
    r.launch = dta::LAUNCH_ROWS;
    r.direct_from = (a->mode == DTA_MODE_DELTA) ? L.n_anchor : 0;
    if (a->anchor_delta_in) {
      // the anchors' deltas are given: the list is the dense tail alone, every
      // row of it stored to out at position s_p + index
      r.n_anchor = 0;
      r.anchors = nullptr;
      r.direct_from = 0;
    }
    r.n_dense_tiles = L.split.n_dense_tiles;
    r.n_sparse_tiles = L.n_sparse_tiles;
    r.split_c = L.split.c;
    r.split_cmax = L.split.cmax;
    r.n_jobs = (r.n_dense_tiles * L.split.cmax + r.n_sparse_tiles) * B * Hkv;
    const int grid = r.n_jobs < sms ? r.n_jobs : sms;
    if ((e = dta::launch_prefill(r, d, grid, false, stream)) != cudaSuccess) return fail_cuda(e);
    rows_launched = true;
  }
  // delta = dense - sparse per anchor (bf16 for the windowed launch, fp32 telemetry on request)
  if ((phases & DTA_PHASE_ROWS) && L.buf_bytes && !fuse) {
    const long long n = (long long)B * L.n_anchor * H * d;
    if ((e = dta::launch_anchor_delta(p.dense_buf, p.sparse_buf, delta_buf, a->anchor_delta, n, stream)) !=
        cudaSuccess)
      return fail_cuda(e);
  }
  // launch 2: windowed rows [0, row_end) with the fused delta epilogue
  if (phases & DTA_PHASE_WINDOW) {
    dta::PrefillParams w = p;
    w.launch = dta::LAUNCH_WINDOW;
    w.fuse_delta = fuse;
    w.delta_cross = L.delta_cross;
    w.win_group = L.win_group;
    w.delta_pair = fuse && G == 4 && a->gamma == 2 * R;
    w.anchor_delta_f32 = fuse ? a->anchor_delta : nullptr;
    // out [B, S, H, d] seen as (d, s, H, B) with a (64, R, G, 1) box: one box is
    // one query tile, rows in the tile's order (head-major), so full tiles
    // leave the kernel with a TMA store; without a map the kernel stores rows
    w.tma_out = encode_4d(&w.tm_out, a->out, d, S, H, B, (long long)H * d, d, (long long)S * H * d, R, G) == DTA_OK;
    w.row_end = (a->mode == DTA_MODE_SPARSE_ONLY) ? S : L.s_p;
    w.n_window_tiles = (w.row_end + JR - 1) / JR;
    w.n_jobs = w.n_window_tiles * B * Hkv;
    if (w.n_jobs > 0) {
      const int groups = w.n_jobs / w.win_group;  // (win_group divides the tiles of every group)
      const int grid = groups < sms ? groups : sms;
      // queued right behind this call's rows launch (or its delta kernel): its
      // CTAs may start on SMs the rows launch no longer needs
      if ((e = dta::launch_prefill(w, d, grid, rows_launched, stream)) != cudaSuccess) return fail_cuda(e);
    }
  }
  // (runs between the two launches, stream-ordered)
  return DTA_OK;
}

}  // extern "C"

namespace {

// Validation and split plan of dta_rows (workspace: header | split counters |
// split partials).
int rows_layout(const dta_rows_args* a, int sms, RowsSplit* S, size_t* ws_bytes) {
  if (!a || a->abi_version != DTA_ABI_VERSION) return DTA_ERR_INVALID_ARG;
  if (a->batch <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->seq_len <= 0 || a->n_rows <= 0 ||
      a->kv_len <= 0)
    return DTA_ERR_SHAPE;
  if (a->head_dim != 64 && a->head_dim != 128) return DTA_ERR_HEAD_DIM;
  if (a->n_heads % a->n_kv_heads != 0) return DTA_ERR_SHAPE;
  const int G = a->n_heads / a->n_kv_heads;
  if (G > 128 || 128 % G != 0) return DTA_ERR_SHAPE;
  if (a->split_tiles < 0) return DTA_ERR_INVALID_ARG;
  const int JR = dta::PREFILL_NQ * (128 / G), n = a->n_rows;
  const long long last_key = a->kv_len - 1;
  // key limits come from a device list: assume them spread over [0, kv_len)
  auto tiles_of = [&](int t) {
    const long long i = (t + 1) * (long long)JR < n ? (t + 1) * (long long)JR : n;
    return (int)(last_key * i / n / dta::PREFILL_BN) + 1;
  };
  *S = plan_rows_split(a->batch * a->n_kv_heads, n, JR, a->head_dim, sms, 0, a->split_tiles, tiles_of);
  *ws_bytes = kHeaderBytes + S->cnt_bytes + S->part_o_bytes + S->part_lse_bytes;
  return DTA_OK;
}

}  // namespace

extern "C" {

size_t dta_rows_workspace_size(const dta_rows_args* a) {
  RowsSplit S;
  size_t bytes = 0;
  if (rows_layout(a, sizing_sms(), &S, &bytes) != DTA_OK) return 0;
  return bytes;
}

int dta_rows(const dta_rows_args* a, void* stream_) {
  RowsSplit S;
  size_t ws_bytes = 0;
  int st = rows_layout(a, 148, &S, &ws_bytes);
  if (st != DTA_OK) return st;
  if (!a->workspace) return DTA_ERR_WORKSPACE;
  if (!a->q || !a->k || !a->v || !a->out || !a->q_rows || !a->kv_limit) return DTA_ERR_INVALID_ARG;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out)) return DTA_ERR_ALIGNMENT;
  if (!stride_ok(a->q_stride_s) || !stride_ok(a->q_stride_h) || !stride_ok(a->q_stride_b) ||
      !stride_ok(a->k_stride_s) || !stride_ok(a->k_stride_h) || !stride_ok(a->k_stride_b) ||
      !stride_ok(a->v_stride_s) || !stride_ok(a->v_stride_h) || !stride_ok(a->v_stride_b))
    return DTA_ERR_STRIDE;
  if (a->wait_cycles < 0 || (a->flags & ~DTA_FLAG_TEST_STALL) != 0) return DTA_ERR_INVALID_ARG;
  if (a->error_word && ((uintptr_t)a->error_word & 3u) != 0) return DTA_ERR_ALIGNMENT;
  int sms = 0;
  if ((st = check_device(&sms)) != DTA_OK) return st;
  if ((st = rows_layout(a, sms, &S, &ws_bytes)) != DTA_OK) return st;
  if (a->workspace_bytes < ws_bytes || !aligned16(a->workspace)) return DTA_ERR_WORKSPACE;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int G = a->n_heads / a->n_kv_heads;
  const int B = a->batch, H = a->n_heads, Hkv = a->n_kv_heads, d = a->head_dim, R = 128 / G;
  dta::PrefillParams p;
  memset(&p, 0, sizeof(p));
  p.q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  p.q_sb = a->q_stride_b; p.q_sh = a->q_stride_h; p.q_ss = a->q_stride_s;
  p.B = B; p.H = H; p.Hkv = Hkv; p.G = G; p.R = R;
  p.scale_log2 = a->scaling * 1.4426950408889634f;
  p.window = 0; p.sink = 0; p.qblock = 64;
  p.gamma = 1; p.s_p = 0; p.n_anchor = 0; p.n_sel = a->n_rows;
  dta::fast_div_params(p.qblock, &p.qblock_mul, &p.qblock_sh);
  dta::fast_div_params(p.gamma, &p.gamma_mul, &p.gamma_sh);
  p.q_rows = a->q_rows;
  p.kv_limit = a->kv_limit;
  p.mode = DTA_MODE_RECOMPUTE;
  p.launch = dta::LAUNCH_ROWS;
  p.direct_from = 0;
  p.out_by_list = 1;
  p.out_rows = a->n_rows;
  p.seq_q = a->seq_len;
  p.kv_len = a->kv_len;
  p.out = reinterpret_cast<__nv_bfloat16*>(a->out);
  p.wait_cycles = a->wait_cycles > 0 ? a->wait_cycles : dta::kWaitTimeoutCycles;
  p.test_stall = (a->flags & DTA_FLAG_TEST_STALL) ? 1 : 0;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  p.counter = reinterpret_cast<int*>(ws);
  p.error = a->error_word ? a->error_word : reinterpret_cast<int*>(ws) + 1;
  uint8_t* cur = ws + kHeaderBytes;
  p.part_cnt = S.cnt_bytes ? reinterpret_cast<int*>(cur) : nullptr;
  cur += S.cnt_bytes;
  p.part_o = S.part_o_bytes ? reinterpret_cast<float*>(cur) : nullptr;
  cur += S.part_o_bytes;
  p.part_lse = S.part_lse_bytes ? reinterpret_cast<float*>(cur) : nullptr;
  p.n_dense_tiles = S.n_dense_tiles;
  p.split_c = S.c;
  p.split_cmax = S.cmax;
  p.n_jobs = p.n_dense_tiles * S.cmax * B * Hkv;
  if ((st = encode_4d(&p.tm_k, a->k, d, a->kv_len, Hkv, B, a->k_stride_s, a->k_stride_h, a->k_stride_b, dta::PREFILL_BN, 1)) !=
      DTA_OK)
    return st;
  if ((st = encode_4d(&p.tm_v, a->v, d, a->kv_len, Hkv, B, a->v_stride_s, a->v_stride_h, a->v_stride_b, dta::PREFILL_BN, 1)) !=
      DTA_OK)
    return st;
  cudaError_t e = cudaMemsetAsync(a->workspace, 0, kHeaderBytes + S.cnt_bytes, stream);
  if (e != cudaSuccess) return fail_cuda(e);
  const int grid = p.n_jobs < sms ? p.n_jobs : sms;
  if ((e = dta::launch_prefill(p, d, grid, false, stream)) != cudaSuccess) return fail_cuda(e);
  return DTA_OK;
}

// Chunking of one key set (dta::DecodeSet).  The dense set tiles [0, n) with
// chunks of C keys.  The sparse set tiles [0, sink) from key 0 and
// [n - window, n) from its first key, so its chunks hold only sparse keys;
// with n <= sink + window it tiles [0, n) like the dense set.
// With a device key count n_keys is the capacity: a capacity of at most
// sink + window keeps every live count all-sparse ([0, n) in n_chunks chunks),
// and above it the sink + window chunks also tile [0, n) for a live count of
// at most sink + window.
// Sink and window beyond the cache mean the whole cache: they are clamped to
// n_keys (the same keys, and no int overflow in sink + window).
static long long decode_sink(const dta_decode_args* a) { return a->sink < a->n_keys ? a->sink : a->n_keys; }
static long long decode_window(const dta_decode_args* a) { return a->window < a->n_keys ? a->window : a->n_keys; }

static void decode_chunking(const dta_decode_args* a, int C, bool sparse, dta::DecodeSet* S) {
  const long long n = a->n_keys, sink = decode_sink(a), window = decode_window(a);
  S->chunk = C;
  S->sparse = sparse ? 1 : 0;
  S->n_chunks = (int)((n + C - 1) / C);
  S->n_sink_chunks = (int)((sink + C - 1) / C);
  const int span = S->n_sink_chunks + (int)((window + C - 1) / C);
  S->n_launched = (!sparse || n <= sink + window) ? S->n_chunks : span;
  if (S->n_launched < 1) S->n_launched = 1;  // no sparse keys: one empty partial
  S->partials = nullptr;
}

// Sparse chunk: the shortest multiple of the 64-key stage whose sink and
// window chunks fit one thread-block cluster of DEC_CLUSTER_TARGET CTAs (merged
// in-cluster, one launch per step), if that chunk is at most
// DEC_SPARSE_CLUSTER_CHUNK_MAX keys; otherwise DEC_SPARSE_CHUNK with the merge
// kernel.  A function of (sink, window) only, so anchor and non-anchor steps,
// and host and device key counts, chunk the sparse set alike.
static int decode_sparse_chunk(const dta_decode_args* a) {
  const long long sink = decode_sink(a), window = decode_window(a);
  for (int C = 64; C <= dta::DEC_SPARSE_CLUSTER_CHUNK_MAX; C += 64)
    if ((sink + C - 1) / C + (window + C - 1) / C <= dta::DEC_CLUSTER_TARGET) return C;
  return dta::DEC_SPARSE_CHUNK;
}

// Dense chunk for `sms` SMs (0: the shortest chunk, whose partials bound the
// workspace of every other choice).
static int decode_dense_chunk(const dta_decode_args* a, int sms) {
  int C = dta::DEC_DENSE_CHUNK_MAX;
  if (sms <= 0) return dta::DEC_DENSE_CHUNK_MIN;
  const long long units = (long long)a->batch * a->n_kv_heads;
  while (C > dta::DEC_DENSE_CHUNK_MIN && units * ((a->n_keys + C - 1) / C) < (long long)sms) C /= 2;
  return C;
}

static int decode_setup(const dta_decode_args* a, dta::DecodeParams* p, int sms) {
  if (!a || a->abi_version != DTA_ABI_VERSION) return DTA_ERR_INVALID_ARG;
  if (a->batch <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_keys <= 0) return DTA_ERR_SHAPE;
  if (a->head_dim != 64 && a->head_dim != 128) return DTA_ERR_HEAD_DIM;
  if (a->n_heads % a->n_kv_heads != 0 || a->n_heads / a->n_kv_heads > 8) return DTA_ERR_SHAPE;
  // the kernels' grid y is batch x KV head (at most 65535)
  if ((long long)a->batch * a->n_kv_heads > 65535) return DTA_ERR_SHAPE;
  if (a->window < 0 || a->sink < 0) return DTA_ERR_INVALID_ARG;
  memset(p, 0, sizeof(*p));
  const int n = a->n_keys;
  p->B = a->batch; p->H = a->n_heads; p->Hkv = a->n_kv_heads; p->G = a->n_heads / a->n_kv_heads;
  p->n_keys = n;
  p->scale_log2 = a->scaling * 1.4426950408889634f;
  p->window = (int)decode_window(a); p->sink = (int)decode_sink(a);
  p->n_keys_dev = a->n_keys_dev;
  // with a device key count the kernels decide this per call
  p->all_sparse = (!a->n_keys_dev && n <= (long long)p->sink + p->window) ? 1 : 0;
  decode_chunking(a, decode_dense_chunk(a, sms), false, &p->set[0]);
  decode_chunking(a, decode_sparse_chunk(a), true, &p->set[1]);
  return DTA_OK;
}

// bytes of one key set's partials
static size_t decode_set_bytes(const dta_decode_args* a, const dta::DecodeSet& S) {
  return align_up((size_t)a->batch * a->n_heads * S.n_launched * (4 + a->head_dim) * 4, 256);
}

// Both key sets' partials, whichever outputs the call asks for, at the
// shortest dense chunk (an upper bound for the chunk dta_decode picks).
size_t dta_decode_workspace_size(const dta_decode_args* a) {
  dta::DecodeParams p;
  if (decode_setup(a, &p, 0) != DTA_OK) return 0;
  return decode_set_bytes(a, p.set[0]) + decode_set_bytes(a, p.set[1]);
}

int dta_decode(const dta_decode_args* a, void* stream_) {
  dta::DecodeParams p;
  int st = decode_setup(a, &p, 0);
  if (st != DTA_OK) return st;
  if (!a->q || !a->k || !a->v || (!a->dense_out && !a->sparse_out)) return DTA_ERR_INVALID_ARG;
  if (a->n_keys_dev && ((uintptr_t)a->n_keys_dev & 3u) != 0) return DTA_ERR_ALIGNMENT;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v)) return DTA_ERR_ALIGNMENT;
  if ((a->dense_out && !aligned16(a->dense_out)) || (a->sparse_out && !aligned16(a->sparse_out)))
    return DTA_ERR_ALIGNMENT;
  if (!stride_ok(a->q_stride_h) || !stride_ok(a->q_stride_b) || !stride_ok(a->k_stride_s) ||
      !stride_ok(a->k_stride_h) || !stride_ok(a->k_stride_b) || !stride_ok(a->v_stride_s) ||
      !stride_ok(a->v_stride_h) || !stride_ok(a->v_stride_b))
    return DTA_ERR_STRIDE;
  const size_t need = dta_decode_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need || !aligned16(a->workspace)) return DTA_ERR_WORKSPACE;
  int sms = 0;
  if ((st = check_device(&sms)) != DTA_OK) return st;
  if ((st = decode_setup(a, &p, sms)) != DTA_OK) return st;  // chunking for this device
  p.q = reinterpret_cast<const __nv_bfloat16*>(a->q);
  p.q_sb = a->q_stride_b; p.q_sh = a->q_stride_h;
  p.k = reinterpret_cast<const __nv_bfloat16*>(a->k);
  p.k_sb = a->k_stride_b; p.k_sh = a->k_stride_h; p.k_ss = a->k_stride_s;
  p.v = reinterpret_cast<const __nv_bfloat16*>(a->v);
  p.v_sb = a->v_stride_b; p.v_sh = a->v_stride_h; p.v_ss = a->v_stride_s;
  p.set[0].partials = reinterpret_cast<float*>(a->workspace);
  p.set[1].partials = reinterpret_cast<float*>(reinterpret_cast<char*>(a->workspace) + decode_set_bytes(a, p.set[0]));
  p.dense_out = reinterpret_cast<__nv_bfloat16*>(a->dense_out);
  p.sparse_out = reinterpret_cast<__nv_bfloat16*>(a->sparse_out);
  cudaError_t e = dta::launch_decode(p, a->head_dim, reinterpret_cast<cudaStream_t>(stream_));
  if (e != cudaSuccess) return fail_cuda(e);
  return DTA_OK;
}

int dta_check_workspace(const void* workspace, void* stream_, int* kernel_code) {
  if (!workspace) return DTA_ERR_INVALID_ARG;
  int word = 0;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  cudaError_t e = cudaMemcpyAsync(&word, reinterpret_cast<const int*>(workspace) + 1, sizeof(int),
                                  cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return fail_cuda(e);
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return fail_cuda(e);
  if (kernel_code) *kernel_code = word;
  return word == 0 ? DTA_OK : DTA_ERR_KERNEL_TIMEOUT;
}

}  // extern "C"
