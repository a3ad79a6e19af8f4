"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and host-side validation returns the documented status
before any CUDA call is made."""

import ctypes
import os
import re

import pytest

from delta_attention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "delta_attention_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(dta_[a-z_]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert sorted(_lib.EXPORTED) == _declared()


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in _declared():
        assert hasattr(L, name), name
    assert L.dta_abi_version() == _lib.ABI_VERSION
    assert L.dta_status_string(5).decode().startswith("gamma")


def _prefill_args(**kw):
    a = _lib.PrefillArgs()
    a.abi_version = _lib.ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.seq_len, a.head_dim = 1, 32, 8, 4096, 128
    fake = 1 << 20  # never dereferenced: validation fails before any CUDA call
    a.q = a.k = a.v = a.out = fake
    a.q_stride_b, a.q_stride_h, a.q_stride_s = 32 * 4096 * 128, 4096 * 128, 128
    a.k_stride_b, a.k_stride_h, a.k_stride_s = 8 * 4096 * 128, 4096 * 128, 128
    a.v_stride_b, a.v_stride_h, a.v_stride_s = 8 * 4096 * 128, 4096 * 128, 128
    a.scaling = 128 ** -0.5
    a.gamma, a.window, a.sink, a.q_block, a.mode = 64, 2048, 128, 64, 0
    for k_, v_ in kw.items():
        setattr(a, k_, v_)
    return a


@pytest.mark.parametrize("override,status", [
    (dict(gamma=48), 5),          # s_p % gamma != 0 (reference reshape would fail)
    (dict(seq_len=100), 5),       # seq_len < cut_n
    (dict(head_dim=96), 6),
    (dict(n_kv_heads=5), 2),
    (dict(n_heads=0), 2),
    (dict(mode=7), 1),
    (dict(abi_version=99), 1),
])
def test_validation_status(override, status):
    L = _lib.lib()
    a = _prefill_args(**override)
    assert L.dta_prefill(ctypes.byref(a), None) == status


def _split_bytes(BG, n_sel, JR, d, sms, tiles_of, factor=3, min_tiles=16):
    """Restates the library's split-K sizing of the rows launch (dta_api.cu
    plan_rows_split): no split while the longest row tile is within 10% of the
    work per SM, else chunks of at most total/(sms*factor) key tiles."""
    ndt = (n_sel + JR - 1) // JR
    T = [tiles_of(t) for t in range(ndt)]
    total = sum(T) * BG
    if max(T) * 10 <= total * 11 // sms:
        return 0, 1
    chunk = max(min_tiles, -(-total // (sms * factor)))
    cmax = -(-max(T) // chunk)
    if cmax <= 1:
        return 0, 1
    al = lambda x: (x + 255) // 256 * 256
    slots = BG * ndt * cmax * 2 * 128
    return al(BG * ndt * 2 * 4 * 4) + al(slots * d * 4) + al(slots * 4), cmax


@pytest.mark.parametrize("heads,kv_heads,split_expected", [(32, 8, False), (4, 1, True)])
def test_workspace_size_query(heads, kv_heads, split_expected):
    """No GPU here: the library sizes for a B200's 148 SMs.  Config 2 on one GPU
    (8 KV groups) is balanced without split-K; one KV group (the per-GPU share
    at 8-GPU strong scaling) splits the long dense row tiles."""
    L = _lib.lib()
    s, gamma = 131072, 64
    a = _prefill_args(seq_len=s, n_heads=heads, n_kv_heads=kv_heads)
    n_anchor = (s - 128) // gamma
    s_p = n_anchor * gamma
    n_sel = n_anchor + 128

    def tiles_of(t):
        i = min((t + 1) * 64, n_sel) - 1
        pos = i * gamma if i < n_anchor else s_p + (i - n_anchor)
        return pos // 128 + 1

    split, cmax = _split_bytes(kv_heads, n_sel, 64, 128, 148, tiles_of)
    assert (cmax > 1) == split_expected
    expect = 256 + split + 2 * ((1 * n_anchor * heads * 128 * 4 + 255) // 256 * 256) \
        + (1 * n_anchor * heads * 128 * 2 + 255) // 256 * 256  # counters+partials, fp32 dense + sparse, bf16 delta
    assert L.dta_prefill_workspace_size(ctypes.byref(a)) == expect
    a.mode = 2  # sparse-only needs only the header
    assert L.dta_prefill_workspace_size(ctypes.byref(a)) == 256
    a.workspace = None
    a.mode = 0
    assert L.dta_prefill(ctypes.byref(a), None) == 7


def test_v2_fields_validated():
    L = _lib.lib()
    a = _prefill_args()
    a.workspace, a.workspace_bytes = 1 << 20, 1 << 30
    a.flags = 4  # unknown flag
    assert L.dta_prefill(ctypes.byref(a), None) == 1
    a.flags, a.wait_cycles = 0, -5
    assert L.dta_prefill(ctypes.byref(a), None) == 1
    a.wait_cycles, a.error_word = 0, (1 << 20) + 2  # not 4-byte aligned
    assert L.dta_prefill(ctypes.byref(a), None) == 4
    a.error_word, a.split_tiles = None, -1
    assert L.dta_prefill(ctypes.byref(a), None) == 1


def test_status_strings_cover_every_status():
    L = _lib.lib()
    for st in _lib.STATUS_NAMES:
        assert L.dta_status_string(st).decode() != "unknown status", st


def test_host_validation_of_lists():
    import torch
    from delta_attention_b200 import ops
    with pytest.raises(ValueError, match="anchors"):
        ops._validate_anchors(torch.tensor([0, 64, 64]), 256, 384)
    with pytest.raises(ValueError, match="anchors"):
        ops._validate_anchors(torch.tensor([1, 64]), 256, 384)
    with pytest.raises(ValueError, match="anchors"):
        ops._validate_anchors(torch.tensor([0, 300]), 256, 384)
    ops._validate_anchors(torch.tensor([0, 5, 255]), 256, 384)
    with pytest.raises(ValueError, match="q_rows"):
        ops._validate_rows(torch.tensor([0, 600]), torch.tensor([0, 1]), 512, 512)
    with pytest.raises(ValueError, match="kv_limit"):
        ops._validate_rows(torch.tensor([0, 1]), torch.tensor([0, 512]), 512, 512)
    with pytest.raises(ValueError, match="non-decreasing"):
        ops._validate_rows(torch.tensor([0, 1]), torch.tensor([5, 4]), 512, 512)
    ops._validate_rows(torch.tensor([0, 1]), torch.tensor([4, 5]), 512, 512)


def test_ops_refuse_cpu_tensors():
    import torch
    from delta_attention_b200 import ops
    q = torch.zeros(1, 4, 256, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.prefill(q, k, k, gamma=64, window=64, sink=16)


def test_anchor_delta_in_needs_explicit_anchors():
    L = _lib.lib()
    a = _prefill_args()
    a.workspace, a.workspace_bytes = 1 << 20, 1 << 30
    a.anchor_delta_in = 1 << 21  # uniform anchors: refused
    assert L.dta_prefill(ctypes.byref(a), None) == 1
    assert L.dta_prefill_workspace_size(ctypes.byref(a)) == 0


def _backward_args(**kw):
    a = _lib.BackwardArgs()
    a.abi_version = _lib.ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.seq_len, a.head_dim = 1, 32, 8, 4096, 128
    fake = 1 << 20  # never dereferenced: validation fails before any CUDA call
    a.q = a.k = a.v = a.out = a.grad_out = a.anchor_delta = a.lse_sparse = a.lse_dense = fake
    a.grad_q = a.grad_k = a.grad_v = fake
    a.q_stride_b, a.q_stride_h, a.q_stride_s = 32 * 4096 * 128, 4096 * 128, 128
    a.k_stride_b, a.k_stride_h, a.k_stride_s = 8 * 4096 * 128, 4096 * 128, 128
    a.v_stride_b, a.v_stride_h, a.v_stride_s = 8 * 4096 * 128, 4096 * 128, 128
    a.scaling = 128 ** -0.5
    a.gamma, a.window, a.sink, a.q_block = 64, 1024, 64, 64
    a.delta_grad_scale = 1.0
    for k_, v_ in kw.items():
        setattr(a, k_, v_)
    return a


@pytest.mark.parametrize("override,status", [
    (dict(gamma=48), 5),          # s_p % gamma != 0
    (dict(seq_len=128), 5),       # no anchor row (s_p = 0)
    (dict(head_dim=96), 6),
    (dict(n_kv_heads=2), 2),      # 16 query heads per KV head: not 1, 2, 4 or 8
    (dict(q_block=0), 1),
    (dict(delta_grad_scale=float("nan")), 1),
    (dict(abi_version=2), 1),
    (dict(workspace_bytes=0), 7),  # (size checked before any pointer use)
])
def test_backward_validation_status(override, status):
    L = _lib.lib()
    a = _backward_args(**override)
    assert L.dta_backward(ctypes.byref(a), None) == status


def test_backward_workspace_size():
    """Header, key-major chunk table, the two passes' output gradients (bf16),
    q of the dense rows, row sums and the dense rows' dQ, fp32 dK / dV; each
    section 256-byte aligned (dta_backward.cu backward_layout)."""
    L = _lib.lib()
    a = _backward_args()
    s, H, Hkv, d, g = 4096, 32, 8, 128, 64
    cut = s % g + max(128, g)
    s_p = s - cut
    n_a, n_sel = s_p // g, s_p // g + cut
    al = lambda x: (x + 255) // 256 * 256
    want = (256 + al((-(-s // 128) + 1) * 4) + al(s_p * H * d * 2) + al(n_sel * H * d * 2) + al(H * n_sel * d * 2)
            + al(H * s * 4) + al(H * n_sel * 4) + al(H * n_a * d * 4) + 2 * al(Hkv * s * d * 4))
    assert L.dta_backward_workspace_size(ctypes.byref(a)) == want
    assert L.dta_backward_workspace_size(ctypes.byref(_backward_args(gamma=48))) == 0


def _decode_args(n, H=32, Hkv=8, d=128, b=1, window=2048, sink=128, dev_count=False):
    a = _lib.DecodeArgs()
    a.abi_version = _lib.ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.n_keys, a.head_dim = b, H, Hkv, n, d
    a.scaling = d ** -0.5
    a.window, a.sink = window, sink
    a.n_keys_dev = (1 << 20) if dev_count else None  # never dereferenced by the size query
    return a


def _sparse_chunk(sink, window, target=9, cmax=512, fallback=256):
    """The sparse key set's chunk (dta_api.cu decode_sparse_chunk): the shortest
    multiple of 64 keys whose sink and window chunks number at most `target`
    (at most `cmax` keys), else `fallback`."""
    for c in range(64, cmax + 1, 64):
        if -(-sink // c) + -(-window // c) <= target:
            return c
    return fallback


@pytest.mark.parametrize("n,window,sink,dev_count", [
    (131072, 2048, 128, False),   # config 2: 256-key sparse chunks, 9 of them
    (131072, 2048, 128, True),    # device key count: the same sparse chunking
    (20000, 4096, 128, False),    # 512-key chunks (9)
    (20000, 8192, 128, False),    # too long for one cluster: 256-key chunks and the merge kernel
    (1500, 512, 1024, False),     # n <= sink + window: the sparse set tiles [0, n)
    (600, 5000, 3, False),        # window past the cache (clamped)
    (777, 100, 7, True),
])
def test_decode_workspace_size(n, window, sink, dev_count):
    """Both key sets' partials, [b, H, launched chunks, 4 + d] fp32 each, 256-byte
    aligned: the dense set at its shortest chunk (256 keys), the sparse set at
    the chunking that depends on (sink, window) only."""
    L = _lib.lib()
    H, d = 32, 128
    al = lambda x: (x + 255) // 256 * 256
    s, w = min(sink, n), min(window, n)
    dense = -(-n // 256)
    c = _sparse_chunk(s, w)
    sparse = -(-n // c) if n <= s + w else -(-s // c) + -(-w // c)
    want = al(H * dense * (4 + d) * 4) + al(H * max(sparse, 1) * (4 + d) * 4)
    assert L.dta_decode_workspace_size(ctypes.byref(_decode_args(n, window=window, sink=sink, dev_count=dev_count))) == want
