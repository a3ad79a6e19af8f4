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
