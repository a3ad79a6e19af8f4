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


def test_workspace_size_query():
    L = _lib.lib()
    a = _prefill_args(seq_len=131072)
    n_anchor = (131072 - 128) // 64
    expect = 256 + 2 * ((1 * n_anchor * 32 * 128 * 4 + 255) // 256 * 256) \
        + (1 * n_anchor * 32 * 128 * 2 + 255) // 256 * 256  # fp32 dense + sparse, bf16 delta
    assert L.dta_prefill_workspace_size(ctypes.byref(a)) == expect
    a.mode = 2  # sparse-only needs only the header
    assert L.dta_prefill_workspace_size(ctypes.byref(a)) == 256
    a.workspace = None
    a.mode = 0
    assert L.dta_prefill(ctypes.byref(a), None) == 7


def test_ops_refuse_cpu_tensors():
    import torch
    from delta_attention_b200 import ops
    q = torch.zeros(1, 4, 256, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.prefill(q, k, k, gamma=64, window=64, sink=16)
