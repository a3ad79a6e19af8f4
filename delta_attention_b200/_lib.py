"""ctypes binding of ``libdelta_attention_b200.so`` (the C ABI declared in
``include/delta_attention_b200.h``).

The library is loaded from the package's in-tree ``_lib/`` directory.  There
is no fallback: if the library is missing or cannot be loaded, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("DTA_LIBRARY") or os.path.join(_HERE, "_lib", "libdelta_attention_b200.so")

ABI_VERSION = 3

DTA_OK = 0
STATUS_NAMES = {
    0: "DTA_OK",
    1: "DTA_ERR_INVALID_ARG",
    2: "DTA_ERR_SHAPE",
    3: "DTA_ERR_STRIDE",
    4: "DTA_ERR_ALIGNMENT",
    5: "DTA_ERR_GAMMA",
    6: "DTA_ERR_HEAD_DIM",
    7: "DTA_ERR_WORKSPACE",
    8: "DTA_ERR_CUDA",
    9: "DTA_ERR_UNSUPPORTED_DEVICE",
    10: "DTA_ERR_KERNEL_TIMEOUT",
    11: "DTA_ERR_SCRATCH_LIMIT",
}

# kernel codes written to the error word (dta_ptx.cuh)
KERNEL_CODES = {
    101: "producer wait ran out",
    102: "MMA issuer wait ran out",
    103: "softmax/epilogue wait ran out",
    104: "tensor-core drain wait ran out",
    105: "a query row or key limit outside the tensors (clamped; output not valid)",
}

# dta_prefill_args.flags / dta_rows_args.flags
FLAG_TEST_STALL = 1

MODES = {"delta": 0, "recompute": 1, "sparse-only": 2}

# symbols declared in include/delta_attention_b200.h
EXPORTED = (
    "dta_prefill_workspace_size",
    "dta_prefill",
    "dta_rows_workspace_size",
    "dta_rows",
    "dta_decode_workspace_size",
    "dta_decode",
    "dta_decode_noalloc",
    "dta_abi_version",
    "dta_status_string",
    "dta_last_cuda_error",
    "dta_check_workspace",
    "dta_backward_workspace_size",
    "dta_backward",
)

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("batch", c_i32), ("n_heads", c_i32), ("n_kv_heads", c_i32), ("seq_len", c_i32), ("head_dim", c_i32),
        ("q", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("q_stride_s", c_i64),
        ("k", c_vp), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_s", c_i64),
        ("v", c_vp), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_s", c_i64),
        ("out", c_vp),
        ("scaling", ctypes.c_float),
        ("gamma", c_i32), ("window", c_i32), ("sink", c_i32), ("q_block", c_i32), ("mode", c_i32),
        ("anchors", c_vp), ("n_anchors", c_i32), ("s_p", c_i32),
        ("anchor_delta", c_vp),
        ("phases", c_i32),
        ("workspace", c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("error_word", c_vp), ("wait_cycles", c_i64), ("flags", c_i32), ("split_tiles", c_i32),
        ("anchor_delta_in", c_vp),
        ("lse_sparse", c_vp), ("lse_dense", c_vp),
    ]


PHASE_ROWS = 1
PHASE_WINDOW = 2


class RowsArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("batch", c_i32), ("n_heads", c_i32), ("n_kv_heads", c_i32), ("seq_len", c_i32), ("head_dim", c_i32),
        ("n_rows", c_i32),
        ("q", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("q_stride_s", c_i64),
        ("k", c_vp), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_s", c_i64),
        ("kv_len", c_i32),
        ("v", c_vp), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_s", c_i64),
        ("q_rows", c_vp), ("kv_limit", c_vp),
        ("out", c_vp),
        ("scaling", ctypes.c_float),
        ("workspace", c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("error_word", c_vp), ("wait_cycles", c_i64), ("flags", c_i32), ("split_tiles", c_i32),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("batch", c_i32), ("n_heads", c_i32), ("n_kv_heads", c_i32), ("n_keys", c_i32), ("head_dim", c_i32),
        ("q", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
        ("k", c_vp), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_s", c_i64),
        ("v", c_vp), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_s", c_i64),
        ("scaling", ctypes.c_float),
        ("window", c_i32), ("sink", c_i32),
        ("dense_out", c_vp), ("sparse_out", c_vp),
        ("workspace", c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("n_keys_dev", c_vp),
    ]


class BackwardArgs(ctypes.Structure):
    _fields_ = [
        ("abi_version", c_i32),
        ("batch", c_i32), ("n_heads", c_i32), ("n_kv_heads", c_i32), ("seq_len", c_i32), ("head_dim", c_i32),
        ("q", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("q_stride_s", c_i64),
        ("k", c_vp), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_s", c_i64),
        ("v", c_vp), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_s", c_i64),
        ("out", c_vp), ("grad_out", c_vp),
        ("anchor_delta", c_vp), ("lse_sparse", c_vp), ("lse_dense", c_vp),
        ("grad_q", c_vp), ("grad_k", c_vp), ("grad_v", c_vp),
        ("scaling", ctypes.c_float),
        ("gamma", c_i32), ("window", c_i32), ("sink", c_i32), ("q_block", c_i32),
        ("delta_grad_scale", ctypes.c_float),
        ("workspace", c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("error_word", c_vp), ("wait_cycles", c_i64),
    ]


class DtaError(RuntimeError):
    """Raised for any non-zero dta_status returned by the library."""

    def __init__(self, status: int, what: str, detail: str = ""):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{what}: {name}" + (f" ({detail})" if detail else ""))


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"delta_attention_b200 native library not built: {LIB_PATH} is missing "
                "(run `python -m delta_attention_b200.build`)")
        L = ctypes.CDLL(LIB_PATH)
        L.dta_prefill_workspace_size.argtypes = [ctypes.POINTER(PrefillArgs)]
        L.dta_prefill_workspace_size.restype = ctypes.c_size_t
        L.dta_prefill.argtypes = [ctypes.POINTER(PrefillArgs), c_vp]
        L.dta_prefill.restype = ctypes.c_int
        L.dta_rows_workspace_size.argtypes = [ctypes.POINTER(RowsArgs)]
        L.dta_rows_workspace_size.restype = ctypes.c_size_t
        L.dta_rows.argtypes = [ctypes.POINTER(RowsArgs), c_vp]
        L.dta_rows.restype = ctypes.c_int
        L.dta_decode_workspace_size.argtypes = [ctypes.POINTER(DecodeArgs)]
        L.dta_decode_workspace_size.restype = ctypes.c_size_t
        L.dta_decode.argtypes = [ctypes.POINTER(DecodeArgs), c_vp]
        L.dta_decode.restype = ctypes.c_int
        L.dta_decode_noalloc.argtypes = [ctypes.POINTER(DecodeArgs), c_vp]
        L.dta_decode_noalloc.restype = ctypes.c_int
        L.dta_abi_version.argtypes = []
        L.dta_abi_version.restype = ctypes.c_int
        L.dta_status_string.argtypes = [ctypes.c_int]
        L.dta_status_string.restype = ctypes.c_char_p
        L.dta_last_cuda_error.argtypes = []
        L.dta_last_cuda_error.restype = ctypes.c_int
        L.dta_check_workspace.argtypes = [c_vp, c_vp, ctypes.POINTER(ctypes.c_int)]
        L.dta_check_workspace.restype = ctypes.c_int
        L.dta_backward_workspace_size.argtypes = [ctypes.POINTER(BackwardArgs)]
        L.dta_backward_workspace_size.restype = ctypes.c_size_t
        L.dta_backward.argtypes = [ctypes.POINTER(BackwardArgs), c_vp]
        L.dta_backward.restype = ctypes.c_int
        if L.dta_abi_version() != ABI_VERSION:
            raise RuntimeError("delta_attention_b200 library ABI mismatch")
        _lib = L
        return L


def check(status: int, what: str) -> None:
    if status != DTA_OK:
        detail = ""
        if status == 8:
            detail = f"cudaError {lib().dta_last_cuda_error()}"
        raise DtaError(status, what, detail)
