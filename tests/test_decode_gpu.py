"""GPU parity of the split-K decode kernel against the CPU oracle."""

import pytest
import torch

from oracle import delta_oracle as orc
from tests._helpers import assert_close

pytestmark = pytest.mark.gpu


def _inputs(n, H=32, Hkv=8, d=128, b=1, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, H, 1, d, generator=g).bfloat16()
    k = torch.randn(b, Hkv, n, d, generator=g).bfloat16()
    v = torch.randn(b, Hkv, n, d, generator=g).bfloat16()
    return q, k, v


@pytest.mark.parametrize("n,H,Hkv,d,b,window,sink", [
    (8192, 32, 8, 128, 1, 2048, 1024),
    (3000, 32, 8, 64, 1, 512, 1024),
    (1500, 8, 1, 128, 2, 512, 1024),   # n <= sink + window: sparse == dense
    (20000, 64, 8, 128, 1, 4096, 128),
    (777, 4, 4, 128, 3, 100, 7),
    (20000, 32, 8, 128, 1, 8192, 128),  # window too long for one cluster: merge kernel
    (5000, 8, 2, 64, 2, 1000, 100),     # window start off the chunk grid
    (600, 8, 2, 128, 1, 5000, 3),       # window longer than the cache
])
def test_decode_dense_and_sparse(n, H, Hkv, d, b, window, sink):
    from delta_attention_b200 import ops
    q, k, v = _inputs(n, H, Hkv, d, b, seed=n)
    dense, sparse = ops.decode(q.cuda(), k.cuda(), v.cuda(), window=window, sink=sink)
    sc = d ** -0.5
    ref_d = orc.dense_decode(q.float(), k.float(), v.float(), sc)
    ref_s = orc.sparse_decode(q.float(), k.float(), v.float(), window, sink, sc)
    assert_close(dense.cpu(), ref_d, f"dense decode n={n}")
    assert_close(sparse.cpu(), ref_s, f"sparse decode n={n}")
    # sparse only (non-anchor step launches only the sink/window chunks)
    none, sparse2 = ops.decode(q.cuda(), k.cuda(), v.cuda(), window=window, sink=sink, want_dense=False)
    assert none is None
    assert torch.equal(sparse2, sparse)
    # dense only (with n <= sink + window it comes from the sparse set's launch)
    dense2, none = ops.decode(q.cuda(), k.cuda(), v.cuda(), window=window, sink=sink, want_sparse=False)
    assert none is None
    assert torch.equal(dense2, dense)


def test_decode_long_cache_uses_long_chunks():
    """A 128K-key cache: the dense key set runs in 4096-key chunks (the length
    the library picks when every SM still gets a CTA) and the sparse set in
    256-key chunks; both must still match the oracle."""
    from delta_attention_b200 import ops
    n, H, Hkv, d, window, sink = 131072, 16, 8, 128, 2048, 128
    q, k, v = _inputs(n, H, Hkv, d, seed=123)
    dense, sparse = ops.decode(q.cuda(), k.cuda(), v.cuda(), window=window, sink=sink)
    sc = d ** -0.5
    assert_close(dense.cpu(), orc.dense_decode(q.float(), k.float(), v.float(), sc), "dense decode n=131072")
    assert_close(sparse.cpu(), orc.sparse_decode(q.float(), k.float(), v.float(), window, sink, sc),
                 "sparse decode n=131072")


@pytest.mark.parametrize("cap,window,sink,d,b", [(6000, 2048, 128, 128, 1), (9000, 4096, 1024, 128, 1),
                                                 (3000, 512, 7, 128, 1), (5000, 1000, 64, 64, 2)])
def test_decode_device_key_count(cap, window, sink, d, b):
    """The live key count read on the device (``n_keys_dev``, the CUDA-graph
    decode path) over a cache of ``cap`` keys gives the rows of a call with
    the host count over the first n keys: the sparse rows bit-identical
    (the sparse chunking depends on sink and window only), the dense rows
    within the oracle tolerance (their chunk follows the cache length)."""
    from delta_attention_b200 import ops
    q, k, v = _inputs(cap, 16, 4, d, b, seed=cap)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    sc = d ** -0.5
    live = torch.zeros(1, dtype=torch.int32, device="cuda")
    for n in sorted({1, 100, sink + window, sink + window + 1, cap // 2, cap - 1, cap}):
        live.fill_(n)
        dense, sparse = ops.decode(qc, kc, vc, window=window, sink=sink, n_keys_dev=live)
        ref_dense, ref_sparse = ops.decode(qc, kc[:, :, :n], vc[:, :, :n], window=window, sink=sink)
        if n > sink + window:
            assert torch.equal(sparse, ref_sparse), f"sparse rows differ at n={n}"
        else:
            assert_close(sparse.cpu(), ref_sparse.cpu().double(), f"sparse n={n}")
        kn, vn = k[:, :, :n].float(), v[:, :, :n].float()
        assert_close(dense.cpu(), orc.dense_decode(q.float(), kn, vn, sc), f"dense decode n={n}")
        assert_close(sparse.cpu(), orc.sparse_decode(q.float(), kn, vn, window, sink, sc), f"sparse decode n={n}")
        _, sparse_only = ops.decode(qc, kc, vc, window=window, sink=sink, n_keys_dev=live, want_dense=False)
        assert torch.equal(sparse_only, sparse)
