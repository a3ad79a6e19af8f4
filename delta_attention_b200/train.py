"""Differentiable delta attention on B200: the drop-in for
``delta_attention/train/flex_delta.py`` (``delta_forward_train``,
``anchor_layout``, ``anchor_grad_ratio``, ``Q_BLOCK``).

The forward is the inference kernel (``dta_prefill``, uniform anchors, delta
mode) run with its log-sum-exp outputs and the fp32 anchor deltas kept; the
backward is ``dta_backward`` (tcgen05 kernels for dK/dV and dQ plus the delta
broadcast's gradient).  Same arguments, output layout ``[b, s, h, d]`` and
ablation arms as the reference (``flex_delta.py:95-196``):
``detach_delta=True`` stops the gradient through the reused correction,
``delta_grad_scale`` scales it.  There is no CPU path.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops

Q_BLOCK = 64  # the reference's block of the block-anchored window (flex_delta.py:48)


def anchor_layout(s: int, gamma: int) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Anchor rows, dense tail rows and s_p (``flex_delta.py:72-76``)."""
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    return torch.arange(0, s_p, gamma), torch.arange(s_p, s), s_p


class _DeltaAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, gamma, window, sink, scaling, delta_grad_scale):
        b, H, s, d = q.shape
        _, _, s_p = anchor_layout(s, gamma)
        n_sel = s_p // gamma + (s - s_p)
        lse_sp = torch.empty(b, H, s, dtype=torch.float32, device=q.device)
        lse_dn = torch.empty(b, H, n_sel, dtype=torch.float32, device=q.device)
        out, delta = ops.prefill(q, k, v, gamma=gamma, window=window, sink=sink, scaling=scaling,
                                 q_block=Q_BLOCK, return_anchor_delta=True, lse_sparse=lse_sp,
                                 lse_dense=lse_dn)
        ctx.save_for_backward(q, k, v, out, delta, lse_sp, lse_dn)
        ctx.cfg = (gamma, window, sink, scaling, delta_grad_scale)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out, delta, lse_sp, lse_dn = ctx.saved_tensors
        gamma, window, sink, scaling, delta_grad_scale = ctx.cfg
        dq, dk, dv = ops.backward(q, k, v, out, grad_out, delta, lse_sp, lse_dn, gamma=gamma, window=window,
                                  sink=sink, scaling=scaling, q_block=Q_BLOCK,
                                  delta_grad_scale=delta_grad_scale)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None, None, None


def delta_forward_train(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gamma: int, window: int,
                        sink: int = 1024, scaling: Optional[float] = None, detach_delta: bool = False,
                        delta_grad_scale: float = 1.0) -> torch.Tensor:
    """Differentiable delta-corrected attention (``flex_delta.py:95-196``).

    q: [b, h, s, d]; k/v: [b, h_kv, s, d] (GQA shared in the kernels, no copy).
    Returns [b, s, h, d].  ``s`` must be a multiple of 64 (the reference's
    block-anchored window is reconciled for whole query blocks only).
    """
    b, h, s, d = q.shape
    if s % Q_BLOCK != 0:
        raise ValueError(f"s={s} must be a multiple of {Q_BLOCK} (block-anchored window semantics are only "
                         "reconciled for full query blocks)")
    if scaling is None:
        scaling = d ** -0.5
    scale = 0.0 if detach_delta else float(delta_grad_scale)
    return _DeltaAttentionFn.apply(q, k, v, int(gamma), int(window), int(sink), float(scaling), scale)


def anchor_grad_ratio(q_grad: torch.Tensor, gamma: int) -> float:
    """Mean per-row gradient norm at dense rows (anchors and tail) over that at
    the other rows (``flex_delta.py:198-210``; a training metric)."""
    s = q_grad.size(2)
    idx, tail, _ = anchor_layout(s, gamma)
    norms = q_grad.float().norm(dim=-1).mean(dim=1)[0]
    is_dense = torch.zeros(s, dtype=torch.bool, device=q_grad.device)
    is_dense[idx.to(q_grad.device)] = True
    is_dense[tail.to(q_grad.device)] = True
    return (norms[is_dense].mean() / norms[~is_dense].mean().clamp_min(1e-12)).item()
