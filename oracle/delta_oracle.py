"""CPU restatement of the reference's delta-attention hot path (TEST ORACLE).

This module is test infrastructure: it is the checker for the CUDA kernels in
``delta_attention_b200`` and the timed CPU reference arm of ``bench.py``.  It
is never imported by the product package.

Everything is written with plain torch CPU tensor ops in float64 (default) so
it is a higher-precision "truth" than the reference's bf16 GPU path.  Every
function cites the reference file:line whose behaviour it restates (paths are
relative to the reference project root).

Semantics restated here
-----------------------
* anchor layout (``cut_n``/``s_p``/anchors/tail):
  ``delta_attention/llama.py:692-693,709-715`` and
  ``delta_attention/train/flex_delta.py:72-76``.
* key-sparse (sink + block-anchored sliding window) attention: the mask of
  ``delta_attention/train/flex_delta.py:59-61`` (hip-attn BLOCKWISE_MASKING
  semantics, window anchored at the last row of each 64-row query block).
* key-dense rows: causal attention of selected rows, row ``i`` attends keys
  ``[0, limit_i]`` (``delta_attention/delta_kernel.py:57-70``, row-masked SDPA
  of ``tests/test_math_identities.py:78-83``).
* delta correction + broadcast: ``delta_attention/llama.py:733-757``;
  modes ``sparse-only`` (``:695-696``) and ``recompute`` (``:725-731``).
* variable-stride correction: ``delta_attention/stride.py:26-40``.
* decode: ``delta_attention/llama.py:498-634``.
* training forward with autograd (the checker of the backward kernels):
  ``delta_attention/train/flex_delta.py:95-196`` including its
  ``detach_delta`` / ``delta_grad_scale`` arms (``_ScaleGrad``, ``:79-93``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch

__all__ = [
    "Q_BLOCK",
    "anchor_layout",
    "sparse_keep",
    "masked_rows_attention",
    "sparse_rows",
    "dense_rows",
    "delta_forward",
    "delta_forward_rows",
    "delta_forward_variable",
    "apply_delta_variable",
    "owner_of_rows",
    "dense_decode",
    "sparse_decode",
    "OracleDecodeState",
    "delta_decode_step",
    "uniform_effective_sparsity",
    "row_cos",
    "delta_forward_train",
]

# hip-attn block_sparse_block_size_q; the window is anchored per block of this
# many query rows (delta_attention/train/flex_delta.py:48, config.py:117,136).
Q_BLOCK = 64


# --------------------------------------------------------------------------
# a1: anchor layout
# --------------------------------------------------------------------------

def anchor_layout(s: int, gamma: int) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Anchor rows, dense-tail rows and ``s_p``.

    ``cut_n = s % gamma + max(128, gamma)``; ``s_p = s - cut_n``; anchors are
    ``arange(0, s_p, gamma)`` and the tail is ``arange(s_p, s)``
    (``delta_attention/llama.py:692-693,709-715``;
    ``delta_attention/train/flex_delta.py:72-76``;
    ``delta_attention/validation.py:224-232``).
    """
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    return torch.arange(0, s_p, gamma), torch.arange(s_p, s), s_p


def uniform_effective_sparsity(s: int, gamma: int, window: int, sink: int = 1024) -> float:
    """Effective sparsity of the fixed-stride layout
    (``delta_attention/stride.py:89-99,115-128``): one minus the causally
    clipped StreamingLLM key count plus the anchor and tail rows' dense key
    counts, over ``s*s/2``."""
    w = min(window + sink, s)
    sparse_cost = w * (w - 1) // 2 + (s - (w - 1)) * w
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    n = (s_p + gamma - 1) // gamma
    anchor_cost = gamma * n * (n - 1) // 2 + n
    tail_cost = (s * (s + 1) - s_p * (s_p + 1)) // 2
    return 1.0 - (sparse_cost + anchor_cost + tail_cost) / (s * s / 2.0)


# --------------------------------------------------------------------------
# a2/a3: masked attention over a set of rows
# --------------------------------------------------------------------------

def sparse_keep(q_idx: torch.Tensor, kv_idx: torch.Tensor, window: int, sink: int,
                q_block: int = Q_BLOCK) -> torch.Tensor:
    """Block-anchored StreamingLLM mask (``delta_attention/train/flex_delta.py:59-61``):
    ``causal AND (kv < sink OR kv + window > block_last(q))`` with
    ``block_last(q) = (q // q_block) * q_block + q_block - 1``."""
    block_last = (q_idx // q_block) * q_block + (q_block - 1)
    return (q_idx >= kv_idx) & ((kv_idx < sink) | (kv_idx + window > block_last))


def masked_rows_attention(q_rows: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          cols: torch.Tensor, keep: torch.Tensor, scaling: float,
                          dtype=torch.float64) -> torch.Tensor:
    """Softmax attention of gathered query rows over a gathered key set.

    q_rows [b, H, n, d]; k, v [b, Hkv, s, d] (GQA: head h uses kv head
    ``h // (H // Hkv)``, as ``repeat_kv`` in ``delta_attention/llama.py:218-229``);
    cols [K] key positions; keep [n, K] bool.  Rows with no kept key produce
    zeros (FlexAttention's convention for fully masked rows).
    Returns [b, n, H, d] in ``dtype``.
    """
    b, H, n, d = q_rows.shape
    Hkv = k.shape[1]
    G = H // Hkv
    qq = q_rows.to(dtype).reshape(b, Hkv, G, n, d)
    kk = k[:, :, cols].to(dtype).unsqueeze(2)  # [b, Hkv, 1, K, d]
    vv = v[:, :, cols].to(dtype).unsqueeze(2)
    scores = torch.matmul(qq, kk.transpose(-1, -2)) * scaling  # [b,Hkv,G,n,K]
    scores = scores.masked_fill(~keep, float("-inf"))
    mx = scores.amax(dim=-1, keepdim=True)
    mx = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    p = torch.exp(scores - mx)
    denom = p.sum(dim=-1, keepdim=True)
    o = torch.matmul(p, vv) / torch.where(denom > 0, denom, torch.ones_like(denom))
    return o.reshape(b, H, n, d).transpose(1, 2)


def _row_chunks(rows: torch.Tensor, chunk: int):
    for i in range(0, rows.numel(), chunk):
        yield i, rows[i:i + chunk]


def sparse_rows(q, k, v, rows, window: int, sink: int, scaling: float,
                q_block: int = Q_BLOCK, dtype=torch.float64, chunk: int = 128) -> torch.Tensor:
    """Key-sparse attention output of the given query rows, [b, n, H, d].

    The reference's sparse branch is hip-attn ``block_sparse_attention`` with an
    empty top-k set (``delta_attention/llama.py:407-449``); its semantics are
    the FlexAttention mask of ``delta_attention/train/flex_delta.py:59-61``,
    pinned to the inference path by the reference's T13
    (``tests/test_flex_delta.py:43-62``).
    """
    rows = torch.as_tensor(rows, dtype=torch.long)
    b, H, s, d = q.shape
    out = torch.empty(b, rows.numel(), H, d, dtype=dtype)
    for i, r in _row_chunks(rows, chunk):
        lo = int(((r.min() // q_block) * q_block + q_block - 1) - window + 1)
        hi = int(r.max())
        win = torch.arange(max(lo, 0), hi + 1)
        snk = torch.arange(0, min(sink, max(lo, 0)))
        cols = torch.cat((snk, win))
        keep = sparse_keep(r[:, None], cols[None, :], window, sink, q_block)
        out[:, i:i + r.numel()] = masked_rows_attention(q[:, :, r], k, v, cols, keep, scaling, dtype)
    return out


def dense_rows(q, k, v, rows, scaling: float, limits=None, dtype=torch.float64,
               chunk: int = 16) -> torch.Tensor:
    """Key-dense causal attention of the given query rows, [b, n, H, d].

    Row ``i`` attends keys ``[0, limits[i]]`` (``limits`` defaults to the row
    index itself), exactly the ``qsa_kernel`` contract of
    ``delta_attention/delta_kernel.py:57-70`` as exercised by
    ``tests/test_math_identities.py:78-83``.
    """
    rows = torch.as_tensor(rows, dtype=torch.long)
    limits = rows if limits is None else torch.as_tensor(limits, dtype=torch.long)
    b, H, s, d = q.shape
    out = torch.empty(b, rows.numel(), H, d, dtype=dtype)
    for i, r in _row_chunks(rows, chunk):
        lim = limits[i:i + r.numel()]
        cols = torch.arange(0, int(lim.max()) + 1)
        keep = cols[None, :] <= lim[:, None]
        out[:, i:i + r.numel()] = masked_rows_attention(q[:, :, r], k, v, cols, keep, scaling, dtype)
    return out


# --------------------------------------------------------------------------
# a4/a5: delta correction, modes
# --------------------------------------------------------------------------

def _check_layout(s: int, gamma: int) -> None:
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    if s_p < 0:
        raise ValueError(f"s={s} shorter than cut_n={cut_n} for gamma={gamma}")
    if s_p % gamma != 0:
        # delta_attention/llama.py:748-749 reshape needs s_p % gamma == 0
        raise ValueError(f"gamma={gamma} does not divide s_p={s_p}")


def delta_forward(q, k, v, gamma: int, window: int, sink: int, scaling: Optional[float] = None,
                  mode: str = "delta", q_block: int = Q_BLOCK, dtype=torch.float64) -> torch.Tensor:
    """Full delta-corrected output [b, s, H, d] (``delta_attention/llama.py:659-757``
    with the sparse branch of ``flex_delta.py:59-61``)."""
    b, H, s, d = q.shape
    if scaling is None:
        scaling = d ** -0.5
    allr = torch.arange(s)
    sparse = sparse_rows(q, k, v, allr, window, sink, scaling, q_block, dtype)
    if mode == "sparse-only":  # llama.py:695-696
        return sparse
    _check_layout(s, gamma)
    anchors, tail, s_p = anchor_layout(s, gamma)
    sel = torch.cat((anchors, tail))
    dense = dense_rows(q, k, v, sel, scaling, dtype=dtype)
    if mode == "recompute":  # llama.py:725-731
        out = torch.zeros(b, s, H, d, dtype=dtype)
        out[:, :s_p] = sparse[:, :s_p]
        out[:, sel] = dense
        return out
    if mode != "delta":
        raise ValueError(f"unknown mode {mode!r}")
    n = anchors.numel()
    delta = dense[:, :n] - sparse[:, anchors]  # llama.py:740
    corrected = (sparse[:, :s_p].reshape(b, n, gamma, H, d)
                 + delta.reshape(b, n, 1, H, d)).reshape(b, s_p, H, d)  # llama.py:748-753
    return torch.cat((corrected, dense[:, n:]), dim=1)  # llama.py:755


def owner_of_rows(anchors: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    """Index (into ``anchors``) of the nearest anchor <= row
    (``delta_attention/stride.py:37``: ``searchsorted(idx, arange, right=True) - 1``)."""
    return torch.searchsorted(anchors, rows, right=True) - 1


def apply_delta_variable(sparse_out, dense_out_sel, idx, s_p: int):
    """Variable-stride correction (``delta_attention/stride.py:26-40``): row i of
    ``sparse_out[:, :s_p]`` gets the delta of the nearest anchor <= i."""
    deltas = dense_out_sel - sparse_out[:, idx]
    owner = owner_of_rows(idx, torch.arange(s_p))
    return sparse_out[:, :s_p] + deltas[:, owner]


def delta_forward_variable(q, k, v, anchors, window: int, sink: int, s_p: int,
                           scaling: Optional[float] = None, q_block: int = Q_BLOCK,
                           dtype=torch.float64) -> torch.Tensor:
    """Delta output for an arbitrary sorted anchor list (first anchor 0) with the
    dense tail ``[s_p, s)``: the composition of ``delta_adaptive_forward``
    (``delta_attention/llama.py:808-824``) once anchors are chosen."""
    b, H, s, d = q.shape
    if scaling is None:
        scaling = d ** -0.5
    anchors = torch.as_tensor(anchors, dtype=torch.long)
    sparse = sparse_rows(q, k, v, torch.arange(s_p), window, sink, scaling, q_block, dtype)
    dense_a = dense_rows(q, k, v, anchors, scaling, dtype=dtype)
    corrected = apply_delta_variable(sparse, dense_a, anchors, s_p)
    tail = dense_rows(q, k, v, torch.arange(s_p, s), scaling, dtype=dtype)
    return torch.cat((corrected, tail), dim=1)


def delta_forward_rows(q, k, v, rows, gamma: int, window: int, sink: int,
                       scaling: Optional[float] = None, mode: str = "delta",
                       q_block: int = Q_BLOCK, dtype=torch.float64) -> torch.Tensor:
    """Output rows ``rows`` of :func:`delta_forward` without computing the rest
    ([b, n, H, d]).  Each output row depends only on its own query row, K/V and
    its anchor, so large-N parity can be checked on a row sample."""
    b, H, s, d = q.shape
    if scaling is None:
        scaling = d ** -0.5
    rows = torch.as_tensor(rows, dtype=torch.long)
    out = torch.empty(b, rows.numel(), H, d, dtype=dtype)
    if mode == "sparse-only":
        return sparse_rows(q, k, v, rows, window, sink, scaling, q_block, dtype)
    _check_layout(s, gamma)
    _, _, s_p = anchor_layout(s, gamma)
    is_tail = rows >= s_p
    if mode == "recompute":
        is_dense = is_tail | (rows % gamma == 0)
    elif mode == "delta":
        is_dense = is_tail
    else:
        raise ValueError(f"unknown mode {mode!r}")
    if is_dense.any():
        out[:, is_dense] = dense_rows(q, k, v, rows[is_dense], scaling, dtype=dtype)
    rest = ~is_dense
    if rest.any():
        r = rows[rest]
        sp = sparse_rows(q, k, v, r, window, sink, scaling, q_block, dtype)
        if mode == "delta":
            a = (r // gamma) * gamma
            ua, inv = torch.unique(a, return_inverse=True)
            da = dense_rows(q, k, v, ua, scaling, dtype=dtype)
            sa = sparse_rows(q, k, v, ua, window, sink, scaling, q_block, dtype)
            sp = sp + (da - sa)[:, inv]
        out[:, rest] = sp
    return out


# --------------------------------------------------------------------------
# a7-a9: decode
# --------------------------------------------------------------------------

def dense_decode(q, k, v, scaling: float, dtype=torch.float64) -> torch.Tensor:
    """One decode row over the whole cache (``delta_attention/llama.py:519-535``
    with s == 1: the ``tril(k - s)`` mask keeps every key).  q [b,H,1,d];
    k, v [b,Hkv,n,d]; returns [b,1,H,d]."""
    n = k.shape[2]
    cols = torch.arange(n)
    keep = torch.ones(1, n, dtype=torch.bool)
    return masked_rows_attention(q, k, v, cols, keep, scaling, dtype)


def sparse_decode(q, k, v, window: int, sink: int, scaling: float, dtype=torch.float64) -> torch.Tensor:
    """StreamingLLM decode row (``delta_attention/llama.py:538-550``): the first
    ``sink`` keys plus the last ``window`` keys, or the whole cache when
    ``n <= sink + window``.  The reference hard-codes ``sink = 1024``."""
    n = k.shape[2]
    if n <= sink + window:
        cols = torch.arange(n)
    else:
        cols = torch.cat((torch.arange(sink), torch.arange(n - window, n)))
    keep = torch.ones(1, cols.numel(), dtype=torch.bool)
    return masked_rows_attention(q, k, v, cols, keep, scaling, dtype)


@dataclass
class OracleDecodeState:
    """Per-layer decode state (``delta_attention/llama.py:573-574``)."""
    last_delta: Optional[torch.Tensor] = None
    steps: int = 0
    last_sparse: Optional[torch.Tensor] = None
    cos_hist: List[float] = field(default_factory=list)


def _cos(a, b) -> float:
    return torch.nn.functional.cosine_similarity(a.flatten().double(), b.flatten().double(), dim=0).item()


def delta_decode_step(state: OracleDecodeState, q, k, v, *, window: int, sink: int, scaling: float,
                      gamma_dec: int = 32, refresh_policy: str = "fixed", drift_threshold: float = 0.95,
                      drift_k: float = 2.0, gamma_dec_max: int = 128, dtype=torch.float64):
    """One delta-decode step (``delta_attention/llama.py:552-634``).

    Returns ``(out [b,1,H,d], anchor: bool)`` and updates ``state`` in place.
    Anchor rules (``:586-606``): first step; ``steps+1 >= gamma_dec_max``;
    fixed policy ``steps+1 >= gamma_dec``; ``drift`` policy ``cos < threshold``;
    ``drift_rel`` policy ``cos < mean - k*std`` of the last 16 (needs >= 8).
    """
    sparse_out = sparse_decode(q, k, v, window, sink, scaling, dtype)
    if state.last_delta is None:
        anchor, cur = True, 0
    else:
        cur = state.steps + 1
        anchor = cur >= int(gamma_dec_max)
        if refresh_policy == "fixed" and cur >= int(gamma_dec):
            anchor = True
        if not anchor and refresh_policy in ("drift", "drift_rel") and state.last_sparse is not None:
            c = _cos(sparse_out, state.last_sparse)
            if refresh_policy == "drift":
                anchor = c < float(drift_threshold)
            else:
                hist = state.cos_hist
                if len(hist) >= 8:
                    mu = sum(hist) / len(hist)
                    sd = (sum((x - mu) ** 2 for x in hist) / len(hist)) ** 0.5
                    anchor = c < mu - float(drift_k) * sd
                hist.append(c)
                del hist[:-16]
    if anchor:
        dense_out = dense_decode(q, k, v, scaling, dtype)
        state.last_delta = dense_out - sparse_out
        state.steps = 0
        out = dense_out
    else:
        out = sparse_out + state.last_delta
        state.steps = cur
    state.last_sparse = sparse_out
    return out, anchor


# --------------------------------------------------------------------------
# metric helper
# --------------------------------------------------------------------------

def row_cos(a, b) -> torch.Tensor:
    """Per-row cosine over flattened (h, d) (``delta_attention/validation.py:215-221``).
    Inputs [b, s, h, d]; returns [b, s]."""
    a32 = a.reshape(a.size(0), a.size(1), -1).double()
    b32 = b.reshape(b.size(0), b.size(1), -1).double()
    return torch.nn.functional.cosine_similarity(a32, b32, dim=-1)


# --------------------------------------------------------------------------
# f4: differentiable training forward (checker of the backward kernels)
# --------------------------------------------------------------------------

class _ScaleGrad(torch.autograd.Function):
    """Identity forward, gradient times a constant backward
    (``delta_attention/train/flex_delta.py:79-93``)."""

    @staticmethod
    def forward(ctx, x, scale):
        ctx.scale = scale
        return x

    @staticmethod
    def backward(ctx, grad):
        return grad * ctx.scale, None


def delta_forward_train(q, k, v, gamma: int, window: int, sink: int = 1024, scaling: Optional[float] = None,
                        detach_delta: bool = False, delta_grad_scale: float = 1.0, q_block: int = Q_BLOCK,
                        dtype=torch.float64) -> torch.Tensor:
    """The composition of ``delta_attention/train/flex_delta.py:95-196`` on this
    module's differentiable primitives: sparse rows for every position, dense
    rows for the anchors and the tail (``:176-186``), delta = dense[anchor] -
    sparse[anchor] (``:188``), detached or gradient-scaled (``:189-192``), and
    the broadcast (``:194-199``).  Autograd through it gives the reference
    gradients for the backward kernels (q, k, v may require grad)."""
    b, H, s, d = q.shape
    if scaling is None:
        scaling = d ** -0.5
    _check_layout(s, gamma)
    sparse = sparse_rows(q, k, v, torch.arange(s), window, sink, scaling, q_block, dtype)
    anchors, tail, s_p = anchor_layout(s, gamma)
    sel = torch.cat((anchors, tail))
    dense = dense_rows(q, k, v, sel, scaling, dtype=dtype)
    n = anchors.numel()
    delta = dense[:, :n] - sparse[:, anchors]
    if detach_delta:
        delta = delta.detach()
    elif delta_grad_scale != 1.0:
        delta = _ScaleGrad.apply(delta, delta_grad_scale)
    corrected = (sparse[:, :s_p].reshape(b, n, gamma, H, d) + delta.reshape(b, n, 1, H, d)).reshape(b, s_p, H, d)
    return torch.cat((corrected, dense[:, n:]), dim=1)
