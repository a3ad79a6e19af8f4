"""dta_decode_noalloc: the decode entry point for callers that cannot allocate
device memory (an engine that already gave all HBM to its own arenas, a program
binding only the C ABI with no device allocator, a loop where cudaMalloc would
synchronize the device).  Its scratch is a static device array shared by every
call, so the test makes two calls in a row and checks each against dta_decode
(which uses a caller workspace).  This file is named to be collected last."""

import ctypes

import pytest
import torch

from delta_attention_b200 import _lib, ops
from tests._helpers import assert_close

pytestmark = pytest.mark.gpu


def _args(q, k, v, window, sink, dense, sparse):
    a = _lib.DecodeArgs()
    a.abi_version = _lib.ABI_VERSION
    b, H, _, d = q.shape
    a.batch, a.n_heads, a.n_kv_heads, a.n_keys, a.head_dim = b, H, k.shape[1], k.shape[2], d
    a.q = q.data_ptr()
    a.q_stride_b, a.q_stride_h = q.stride(0), q.stride(1)
    a.k = k.data_ptr()
    a.k_stride_b, a.k_stride_h, a.k_stride_s = k.stride(0), k.stride(1), k.stride(2)
    a.v = v.data_ptr()
    a.v_stride_b, a.v_stride_h, a.v_stride_s = v.stride(0), v.stride(1), v.stride(2)
    a.scaling = d ** -0.5
    a.window, a.sink = window, sink
    a.dense_out = None if dense is None else dense.data_ptr()
    a.sparse_out = sparse.data_ptr()
    return a


def _inputs(seed, b, n):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, 32, 1, 128, generator=g).bfloat16().cuda()
    k = torch.randn(b, 8, n, 128, generator=g).bfloat16().cuda()
    v = torch.randn(b, 8, n, 128, generator=g).bfloat16().cuda()
    return q, k, v


def test_noalloc_decode_matches_workspace_decode_two_calls():
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row with different shapes: the second reuses the array the
    # first left behind
    for seed, b, n, want_dense in ((0, 2, 20000, True), (1, 1, 7000, False)):
        q, k, v = _inputs(seed, b, n)
        ref_d, ref_s = ops.decode(q, k, v, window=2048, sink=1024, want_dense=want_dense)
        dense = torch.empty(b, 1, 32, 128, dtype=torch.bfloat16, device="cuda") if want_dense else None
        sparse = torch.empty(b, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
        a = _args(q, k, v, 2048, 1024, dense, sparse)
        assert lib.dta_decode_noalloc(ctypes.byref(a), ctypes.c_void_p(stream)) == _lib.DTA_OK
        torch.cuda.synchronize()
        assert_close(sparse.cpu(), ref_s.cpu(), f"no-alloc sparse (call seed {seed})")
        if want_dense:
            assert_close(dense.cpu(), ref_d.cpu(), f"no-alloc dense (call seed {seed})")


def test_noalloc_rejects_requests_beyond_its_scratch():
    lib = _lib.lib()
    q, k, v = _inputs(2, 1, 600)
    a = _args(q, k, v, 2048, 1024, None, torch.empty(1, 1, 32, 128, dtype=torch.bfloat16, device="cuda"))
    a.batch = 64
    a.n_keys = 1 << 20  # 64 x 32 heads x 2048 chunks of partials: far beyond 32 MiB
    assert lib.dta_decode_workspace_size(ctypes.byref(a)) > (32 << 20)
    assert lib.dta_decode_noalloc(ctypes.byref(a), None) == 11  # DTA_ERR_SCRATCH_LIMIT
