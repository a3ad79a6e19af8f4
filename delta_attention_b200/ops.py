"""Torch-facing wrappers over the C ABI (device memory, streams and strides).

Each op checks its inputs, sizes the caller-side workspace with the library's
``*_workspace_size`` query, passes raw pointers plus the current CUDA stream,
and raises :class:`DtaError` for any non-zero status.  There is no CPU path.

Kernel-side failures (a bounded wait that ran out, a row index outside the
tensors) cannot be returned by an asynchronous launch.  Every prefill and rows
launch therefore records them in one persistent int32 "error word" per device,
which stays set until :func:`check_errors` reads it (at a point where the
caller synchronises anyway) and raises ``DtaError(DTA_ERR_KERNEL_TIMEOUT)``.
``check=True`` on an op does that right after the launch.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import ABI_VERSION, KERNEL_CODES, BackwardArgs, DecodeArgs, DtaError, PrefillArgs, RowsArgs, lib
from ._lib import check as _check_status

DTA_ERR_KERNEL_TIMEOUT = 10

_error_words = {}


def _device_index(device=None) -> int:
    if device is None:
        return torch.cuda.current_device()
    d = torch.device(device)
    return d.index if d.index is not None else torch.cuda.current_device()


def error_word(device=None) -> torch.Tensor:
    """The persistent device int32 that this device's kernels report into."""
    idx = _device_index(device)
    w = _error_words.get(idx)
    if w is None:
        w = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _error_words[idx] = w
    return w


def check_errors(device=None) -> None:
    """Synchronise the current stream, read this device's error word and raise
    ``DtaError`` (status DTA_ERR_KERNEL_TIMEOUT) if any launch since the last
    check recorded a kernel code; the word is cleared either way."""
    w = error_word(device)
    code = int(w[0].item())  # synchronises with the current stream
    if code != 0:
        w.zero_()
        raise DtaError(DTA_ERR_KERNEL_TIMEOUT, "kernel error word",
                       f"code {code}: {KERNEL_CODES.get(code, 'unknown')}")


def _validate_anchors(anchors: torch.Tensor, s_p: int, s: int) -> None:
    a = anchors.detach().to("cpu", torch.int64)
    if a.numel() == 0 or not 0 < s_p <= s:
        raise ValueError(f"need at least one anchor and 0 < s_p <= seq_len (s_p={s_p}, seq_len={s})")
    if int(a[0]) != 0 or int(a[-1]) >= s_p or (a.numel() > 1 and not bool((a[1:] > a[:-1]).all())):
        raise ValueError("anchors must start at 0, be strictly increasing and lie below s_p")


def _validate_rows(q_rows: torch.Tensor, kv_limit: torch.Tensor, seq_len: int, kv_len: int) -> None:
    r = q_rows.detach().to("cpu", torch.int64)
    lim = kv_limit.detach().to("cpu", torch.int64)
    if r.shape != lim.shape:
        raise ValueError("q_rows and kv_limit must have the same length")
    if bool((r < 0).any()) or bool((r >= seq_len).any()):
        raise ValueError(f"q_rows must lie in [0, {seq_len})")
    if bool((lim < 0).any()) or bool((lim >= kv_len).any()):
        raise ValueError(f"kv_limit must lie in [0, {kv_len})")
    if lim.numel() > 1 and not bool((lim[1:] >= lim[:-1]).all()):
        raise ValueError("kv_limit must be non-decreasing")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _bf16_lastdim_contig(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    if t.stride(-1) != 1 or t.data_ptr() % 16 != 0 or any(
            (s * 2) % 16 != 0 for s in t.stride()[:-1]):
        t = t.contiguous()
    return t


def _strides(t: torch.Tensor):
    """Element strides of the leading dims; size-1 dims get a harmless legal stride."""
    out = []
    for size, st in zip(t.shape[:-1], t.stride()[:-1]):
        if size == 1 or st <= 0:
            st = t.shape[-1]
        out.append(int(st))
    return out


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("delta_attention_b200 ops take CUDA tensors (there is no CPU path)")


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, gamma: int, window: int, sink: int,
            scaling: Optional[float] = None, mode: str = "delta", q_block: int = 64,
            anchors: Optional[torch.Tensor] = None, s_p: Optional[int] = None,
            return_anchor_delta: bool = False, workspace: Optional[torch.Tensor] = None,
            phases: int = 0, out: Optional[torch.Tensor] = None, check: bool = False,
            validate: bool = True, wait_cycles: int = 0, flags: int = 0, split_tiles: int = 0,
            use_error_word: bool = True, anchor_delta_in: Optional[torch.Tensor] = None,
            lse_sparse: Optional[torch.Tensor] = None, lse_dense: Optional[torch.Tensor] = None):
    """Delta-attention prefill of one layer.

    q [b, H, s, d], k/v [b, Hkv, s, d] (post-RoPE; any strides with d
    contiguous).  Returns ``out`` [b, s, H, d] in q's dtype (computation in
    bf16, as the reference's sparse path does, ``delta_attention/llama.py:383-388``),
    and, with ``return_anchor_delta``, the fp32 anchor deltas [b, n_anchor, H, d].
    An explicit ``anchors`` list is checked on the host (``validate``; it
    must start at 0, increase strictly and stay below ``s_p``).  ``check``
    synchronises and raises if a kernel recorded an error (see
    :func:`check_errors`); ``wait_cycles``, ``flags`` and ``split_tiles`` are
    the C ABI's (0 = defaults).  With ``use_error_word=False`` kernel codes go
    to the workspace header instead (read with :func:`check_workspace`).
    ``anchor_delta_in`` [b, n_anchors, H, d] (explicit anchors only): the
    anchors' dense - sparse rows computed earlier; only the dense tail rows
    are then computed again.
    ``lse_sparse`` [b, H, s] and ``lse_dense`` [b, H, n_sel] (fp32, contiguous,
    optional) receive the base-2 log-sum-exp of every windowed row (rows below
    s_p) and of every dense row (anchors, then the tail), which the training
    backward needs.
    """
    _check_cuda(q, k, v)
    odt = q.dtype
    qb, kb, vb = _bf16_lastdim_contig(q), _bf16_lastdim_contig(k), _bf16_lastdim_contig(v)
    b, H, s, d = qb.shape
    Hkv = kb.shape[1]
    if kb.shape != (b, Hkv, s, d) or vb.shape != kb.shape:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if scaling is None:
        scaling = d ** -0.5
    if mode not in _lib.MODES:
        raise ValueError(f"unknown mode {mode!r}")
    if out is None:
        out = torch.empty(b, s, H, d, dtype=torch.bfloat16, device=q.device)
    a = PrefillArgs()
    a.abi_version = ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.seq_len, a.head_dim = b, H, Hkv, s, d
    a.q = _ptr(qb)
    a.q_stride_b, a.q_stride_h, a.q_stride_s = _strides(qb)
    a.k = _ptr(kb)
    a.k_stride_b, a.k_stride_h, a.k_stride_s = _strides(kb)
    a.v = _ptr(vb)
    a.v_stride_b, a.v_stride_h, a.v_stride_s = _strides(vb)
    a.out = _ptr(out)
    a.scaling = float(scaling)
    a.gamma, a.window, a.sink, a.q_block = int(gamma), int(window), int(sink), int(q_block)
    a.mode = _lib.MODES[mode]
    a.phases = int(phases)
    a.split_tiles = int(split_tiles)
    anc = None
    if anchor_delta_in is not None and anchors is None:
        raise ValueError("anchor_delta_in needs explicit anchors")
    if anchors is not None:
        if s_p is None:
            raise ValueError("explicit anchors need s_p")
        if validate:
            _validate_anchors(anchors, int(s_p), s)
        anc = anchors.to(device=q.device, dtype=torch.int32).contiguous()
        a.anchors = _ptr(anc)
        if anchor_delta_in is not None:
            if tuple(anchor_delta_in.shape) != (b, anc.numel(), H, d):
                raise ValueError(f"anchor_delta_in must be [{b}, {anc.numel()}, {H}, {d}]")
            din = anchor_delta_in.to(device=q.device, dtype=torch.bfloat16).contiguous()
            a.anchor_delta_in = _ptr(din)
        a.n_anchors = anc.numel()
        a.s_p = int(s_p)
    ws_bytes = lib().dta_prefill_workspace_size(ctypes.byref(a))
    if ws_bytes == 0:
        # let dta_prefill report the precise validation status
        _check_status(lib().dta_prefill(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_prefill")
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = _workspace(ws_bytes, q.device)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel()
    a.error_word = _ptr(error_word(q.device)) if use_error_word else None
    a.wait_cycles = int(wait_cycles)
    a.flags = int(flags)
    for name, t in (("lse_sparse", lse_sparse), ("lse_dense", lse_dense)):
        if t is not None:
            if t.dtype != torch.float32 or not t.is_contiguous() or t.device != q.device:
                raise ValueError(f"{name} must be a contiguous fp32 tensor on {q.device}")
            setattr(a, name, _ptr(t))
    if lse_sparse is not None and tuple(lse_sparse.shape) != (b, H, s):
        raise ValueError(f"lse_sparse must be [{b}, {H}, {s}]")
    delta = None
    if return_anchor_delta and mode == "delta":
        if anc is not None:
            n_anchor = anc.numel()
        else:
            cut_n = s % gamma + max(128, gamma)
            n_anchor = max(s - cut_n, 0) // gamma
        delta = torch.empty(b, n_anchor, H, d, dtype=torch.float32, device=q.device)
        a.anchor_delta = _ptr(delta)
    _check_status(lib().dta_prefill(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_prefill")
    if check:
        check_errors(q.device)
    if odt != torch.bfloat16:
        out = out.to(odt)
    return (out, delta) if return_anchor_delta else out


def prefill_workspace(batch: int, n_heads: int, n_kv_heads: int, seq_len: int, head_dim: int, *, gamma: int,
                      window: int = 0, sink: int = 0, mode: str = "delta", n_anchors: Optional[int] = None,
                      s_p: Optional[int] = None, split_tiles: int = 0, device=None) -> torch.Tensor:
    """A device workspace of the size ``dta_prefill_workspace_size`` reports, for
    callers that keep one workspace across calls (on the current device; pass
    the window and sink of the calls it will serve)."""
    a = PrefillArgs()
    a.abi_version = ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.seq_len, a.head_dim = batch, n_heads, n_kv_heads, seq_len, head_dim
    a.gamma, a.window, a.sink, a.q_block, a.mode = int(gamma), int(window), int(sink), 64, _lib.MODES[mode]
    a.split_tiles = int(split_tiles)
    if n_anchors is not None:
        a.anchors, a.n_anchors, a.s_p = 16, int(n_anchors), int(s_p)
    nbytes = lib().dta_prefill_workspace_size(ctypes.byref(a))
    if nbytes == 0:
        raise ValueError("invalid prefill arguments for a workspace")
    return _workspace(nbytes, device)


def anchor_deltas(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows: torch.Tensor, *, window: int,
                  sink: int, scaling: Optional[float] = None, q_block: int = 64,
                  validate: bool = True) -> torch.Tensor:
    """dense - sparse (fp32) at the given sorted query rows, [b, n, H, d].

    Runs only the row launch of the prefill (dense and sparse attention of the
    listed rows); used by the adaptive stride planner."""
    s = q.shape[2]
    if validate:
        r = rows.detach().to("cpu", torch.int64)
        if r.numel() == 0 or int(r.min()) < 0 or int(r.max()) >= s or \
                (r.numel() > 1 and not bool((r[1:] > r[:-1]).all())):
            raise ValueError(f"rows must be strictly increasing and lie in [0, {s})")
    rows = rows.to(device=q.device, dtype=torch.int32)
    # no tail rows (s_p == s) and no windowed launch: `out` is never written
    dummy = torch.empty(16, dtype=torch.bfloat16, device=q.device)
    _, delta = prefill(q, k, v, gamma=1, window=window, sink=sink, scaling=scaling, mode="delta",
                       q_block=q_block, anchors=rows, s_p=s, return_anchor_delta=True,
                       phases=_lib.PHASE_ROWS, out=dummy, validate=False)
    return delta


def rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_rows: torch.Tensor, kv_limit: torch.Tensor,
         scaling: Optional[float] = None, *, check: bool = False, validate: bool = True,
         wait_cycles: int = 0, flags: int = 0, split_tiles: int = 0) -> torch.Tensor:
    """Attention for a list of query rows: row i uses ``q[:, :, q_rows[i]]`` and
    attends keys ``[0, kv_limit[i]]`` (non-decreasing).  Returns [b, n, H, d]
    (the ``qsa_kernel`` contract, ``delta_attention/delta_kernel.py:259-329``).
    The lists are checked on the host unless ``validate`` is False."""
    _check_cuda(q, k, v)
    odt = q.dtype
    qb, kb, vb = _bf16_lastdim_contig(q), _bf16_lastdim_contig(k), _bf16_lastdim_contig(v)
    b, H, sq, d = qb.shape
    Hkv, skv = kb.shape[1], kb.shape[2]
    if scaling is None:
        scaling = d ** -0.5
    if validate:
        _validate_rows(q_rows, kv_limit, sq, skv)
    qr = q_rows.to(device=q.device, dtype=torch.int32).contiguous()
    kl = kv_limit.to(device=q.device, dtype=torch.int32).contiguous()
    n = qr.numel()
    out = torch.empty(b, n, H, d, dtype=torch.bfloat16, device=q.device)
    a = RowsArgs()
    a.abi_version = ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.seq_len, a.head_dim, a.n_rows = b, H, Hkv, sq, d, n
    a.q = _ptr(qb)
    a.q_stride_b, a.q_stride_h, a.q_stride_s = _strides(qb)
    a.k = _ptr(kb)
    a.k_stride_b, a.k_stride_h, a.k_stride_s = _strides(kb)
    a.kv_len = skv
    a.v = _ptr(vb)
    a.v_stride_b, a.v_stride_h, a.v_stride_s = _strides(vb)
    a.q_rows, a.kv_limit = _ptr(qr), _ptr(kl)
    a.out = _ptr(out)
    a.scaling = float(scaling)
    a.error_word = _ptr(error_word(q.device))
    a.wait_cycles = int(wait_cycles)
    a.flags = int(flags)
    a.split_tiles = int(split_tiles)
    ws_bytes = lib().dta_rows_workspace_size(ctypes.byref(a))
    if ws_bytes == 0:
        _check_status(lib().dta_rows(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_rows")
    ws = _workspace(ws_bytes, q.device)
    a.workspace, a.workspace_bytes = _ptr(ws), ws.numel()
    _check_status(lib().dta_rows(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_rows")
    if check:
        check_errors(q.device)
    return out if odt == torch.bfloat16 else out.to(odt)


_decode_ws = {}


def _decode_workspace(nbytes: int, device) -> torch.Tensor:
    """Decode workspace kept per (device, stream) and grown on demand: decode
    runs once per layer and token, so a fresh allocation per call would cost
    more host time than the kernel.  Calls on one stream are ordered, so they
    may share it.  (During CUDA graph capture a private buffer is used.)"""
    if torch.cuda.is_current_stream_capturing():
        return _workspace(nbytes, device)
    key = (_device_index(device), _stream())
    ws = _decode_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = _workspace(nbytes, device)
        _decode_ws[key] = ws
    return ws


def decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, window: int, sink: int,
           scaling: Optional[float] = None, want_dense: bool = True, want_sparse: bool = True,
           n_keys: Optional[int] = None, n_keys_dev: Optional[torch.Tensor] = None,
           ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
    """One decode row per (batch, head).  q [b, H, 1, d]; k/v [b, Hkv, n, d]
    (only the first ``n_keys`` keys are used).  Returns ``(dense, sparse)``,
    each [b, 1, H, d] bf16 or None; both come from one pass over the cache.
    ``n_keys_dev`` (a device int32 scalar tensor) gives the live key count on
    the device instead: k/v are then the whole cache (its capacity sizes the
    launch), so a CUDA graph can replay the call while the cache grows."""
    _check_cuda(q, k, v)
    qb, kb, vb = _bf16_lastdim_contig(q), _bf16_lastdim_contig(k), _bf16_lastdim_contig(v)
    b, H, one, d = qb.shape
    if one != 1:
        raise ValueError("decode takes one query row per (batch, head)")
    Hkv, n = kb.shape[1], kb.shape[2] if n_keys is None else int(n_keys)
    if scaling is None:
        scaling = d ** -0.5
    dense = torch.empty(b, 1, H, d, dtype=torch.bfloat16, device=q.device) if want_dense else None
    sparse = torch.empty(b, 1, H, d, dtype=torch.bfloat16, device=q.device) if want_sparse else None
    a = DecodeArgs()
    a.abi_version = ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.n_keys, a.head_dim = b, H, Hkv, n, d
    a.q = _ptr(qb)
    a.q_stride_b, a.q_stride_h = _strides(qb)[:2]
    a.k = _ptr(kb)
    a.k_stride_b, a.k_stride_h, a.k_stride_s = _strides(kb)
    a.v = _ptr(vb)
    a.v_stride_b, a.v_stride_h, a.v_stride_s = _strides(vb)
    a.scaling = float(scaling)
    a.window, a.sink = int(window), int(sink)
    a.dense_out, a.sparse_out = _ptr(dense), _ptr(sparse)
    if n_keys_dev is not None:
        if n_keys_dev.dtype != torch.int32 or n_keys_dev.device != q.device or n_keys_dev.numel() != 1:
            raise ValueError("n_keys_dev must be a one-element int32 tensor on q's device")
        a.n_keys, a.n_keys_dev = kb.shape[2], _ptr(n_keys_dev)
    ws = _decode_workspace(lib().dta_decode_workspace_size(ctypes.byref(a)), q.device)
    a.workspace, a.workspace_bytes = _ptr(ws), ws.numel()
    _check_status(lib().dta_decode(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_decode")
    return dense, sparse


def backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, grad_out: torch.Tensor,
             anchor_delta: torch.Tensor, lse_sparse: torch.Tensor, lse_dense: torch.Tensor, *, gamma: int,
             window: int, sink: int, scaling: Optional[float] = None, q_block: int = 64,
             delta_grad_scale: float = 1.0, check: bool = False, wait_cycles: int = 0):
    """Gradients (dq, dk, dv), bf16, of the delta-attention layer with uniform
    anchors (``dta_backward``): q [b, H, s, d], k/v [b, Hkv, s, d] and the
    forward's ``out`` [b, s, H, d], fp32 ``anchor_delta`` [b, n_anchor, H, d],
    ``lse_sparse`` [b, H, s] and ``lse_dense`` [b, H, n_sel] (from
    :func:`prefill` with the same parameters); ``grad_out`` [b, s, H, d].
    ``delta_grad_scale`` multiplies the gradient through the broadcast delta
    (0 = the delta detached)."""
    _check_cuda(q, k, v, out, grad_out, anchor_delta, lse_sparse, lse_dense)
    qb, kb, vb = _bf16_lastdim_contig(q), _bf16_lastdim_contig(k), _bf16_lastdim_contig(v)
    b, H, s, d = qb.shape
    Hkv = kb.shape[1]
    if kb.shape != (b, Hkv, s, d) or vb.shape != kb.shape:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if tuple(out.shape) != (b, s, H, d) or tuple(grad_out.shape) != (b, s, H, d):
        raise ValueError("out and grad_out must be [b, s, H, d]")
    if scaling is None:
        scaling = d ** -0.5
    ob = out.to(torch.bfloat16).contiguous()
    gb = grad_out.to(torch.bfloat16).contiguous()
    ad = anchor_delta.to(torch.float32).contiguous()
    ls = lse_sparse.to(torch.float32).contiguous()
    ld = lse_dense.to(torch.float32).contiguous()
    dq = torch.empty(b, H, s, d, dtype=torch.bfloat16, device=q.device)
    dk = torch.empty(b, Hkv, s, d, dtype=torch.bfloat16, device=q.device)
    dv = torch.empty_like(dk)
    a = BackwardArgs()
    a.abi_version = ABI_VERSION
    a.batch, a.n_heads, a.n_kv_heads, a.seq_len, a.head_dim = b, H, Hkv, s, d
    a.q = _ptr(qb)
    a.q_stride_b, a.q_stride_h, a.q_stride_s = _strides(qb)
    a.k = _ptr(kb)
    a.k_stride_b, a.k_stride_h, a.k_stride_s = _strides(kb)
    a.v = _ptr(vb)
    a.v_stride_b, a.v_stride_h, a.v_stride_s = _strides(vb)
    a.out, a.grad_out = _ptr(ob), _ptr(gb)
    a.anchor_delta, a.lse_sparse, a.lse_dense = _ptr(ad), _ptr(ls), _ptr(ld)
    a.grad_q, a.grad_k, a.grad_v = _ptr(dq), _ptr(dk), _ptr(dv)
    a.scaling = float(scaling)
    a.gamma, a.window, a.sink, a.q_block = int(gamma), int(window), int(sink), int(q_block)
    a.delta_grad_scale = float(delta_grad_scale)
    ws_bytes = lib().dta_backward_workspace_size(ctypes.byref(a))
    if ws_bytes == 0:
        _check_status(lib().dta_backward(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_backward")
    workspace = _workspace(ws_bytes, q.device)
    a.workspace = _ptr(workspace)
    a.workspace_bytes = workspace.numel()
    a.error_word = _ptr(error_word(q.device))
    a.wait_cycles = int(wait_cycles)
    _check_status(lib().dta_backward(ctypes.byref(a), ctypes.c_void_p(_stream())), "dta_backward")
    if check:
        check_errors(q.device)
    return dq, dk, dv


def check_workspace(workspace: torch.Tensor) -> int:
    """Synchronously read a workspace's kernel error word; raises on a timeout."""
    code = ctypes.c_int(0)
    st = lib().dta_check_workspace(ctypes.c_void_p(_ptr(workspace)), ctypes.c_void_p(_stream()),
                                   ctypes.byref(code))
    _check_status(st, f"kernel error word {code.value}")
    return code.value
