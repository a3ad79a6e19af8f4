"""Variable-stride anchors and the adaptive stride planner.

Restates the host policy of ``delta_attention/stride.py`` (stride update
rules ``next_gamma`` / ``next_gamma_relative`` ``:55-86``, chunking ``:111-112``,
cost model ``:89-128``) and drives the kernels for the chunked adaptive
placement of ``delta_attention/llama.py:759-824``: per chunk, the anchor
deltas come from the prefill's row launch (``ops.anchor_deltas``); the final
output is one ``ops.prefill`` call with the chosen anchor list and those
deltas (so no anchor row is computed twice), whose windowed launch applies
the variable-stride broadcast (row i gets the delta of the nearest anchor <= i,
``delta_attention/stride.py:26-40``) in its epilogue.
"""

from __future__ import annotations

from typing import Any, Dict, List, Tuple

import torch

from . import ops

ADAPT_MARGIN = 0.02  # hysteresis above adapt_threshold before growing gamma


def plan_chunks(s_p: int, chunk: int) -> List[Tuple[int, int]]:
    return [(a, min(a + chunk, s_p)) for a in range(0, s_p, chunk)]


def next_gamma(cos_mean: float, gamma_c: int, *, threshold: float, gamma_min: int, gamma_max: int) -> int:
    """Halve on fast drift (cos below threshold), double when smooth (above threshold + margin)."""
    if cos_mean < threshold:
        return max(gamma_c // 2, gamma_min)
    if cos_mean > threshold + ADAPT_MARGIN:
        return min(gamma_c * 2, gamma_max)
    return gamma_c


def next_gamma_relative(cos_mean: float, history: List[float], gamma_c: int, *, k: float,
                        gamma_min: int, gamma_max: int) -> int:
    """Halve/double on deviations beyond k std from the running mean of earlier
    chunks; needs at least two history entries."""
    if len(history) < 2:
        return gamma_c
    mu = sum(history) / len(history)
    sd = (sum((x - mu) ** 2 for x in history) / len(history)) ** 0.5
    if cos_mean < mu - k * sd:
        return max(gamma_c // 2, gamma_min)
    if cos_mean > mu + k * sd:
        return min(gamma_c * 2, gamma_max)
    return gamma_c


def interanchor_cos(deltas: torch.Tensor) -> Tuple[float, float]:
    """(mean, min) cosine between consecutive anchor deltas; deltas [b, n, h, d]."""
    if deltas.size(1) < 2:
        return 1.0, 1.0
    cos = torch.nn.functional.cosine_similarity(deltas[:, :-1].float(), deltas[:, 1:].float(), dim=-1)
    return cos.mean().item(), cos.min().item()


def sparse_pass_cost(s: int, window: int, sink: int) -> int:
    """Causally clipped StreamingLLM key count: row i attends min(i+1, window+sink) keys."""
    w = min(window + sink, s)
    return w * (w - 1) // 2 + (s - (w - 1)) * w


def effective_sparsity(anchor_idx, s: int, window: int, sink: int = 1024) -> float:
    """1 - (clipped sparse cost + sum of anchor/tail row costs) / (s^2/2)."""
    idx = torch.as_tensor(anchor_idx)
    dense_cost = int(idx.sum().item()) + idx.numel()
    return 1.0 - (sparse_pass_cost(s, window, sink) + dense_cost) / (s * s / 2.0)


def uniform_effective_sparsity(s: int, gamma: int, window: int, sink: int = 1024) -> float:
    """Effective sparsity of the fixed layout (anchors + cut_n tail)."""
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    n = (s_p + gamma - 1) // gamma
    anchor_cost = gamma * n * (n - 1) // 2 + n
    tail_cost = (s * (s + 1) - s_p * (s_p + 1)) // 2
    return 1.0 - (sparse_pass_cost(s, window, sink) + anchor_cost + tail_cost) / (s * s / 2.0)


def adaptive_prefill(cfg, q, k, v, scaling, layer_idx: int = 0):
    """Chunked adaptive anchor placement; returns (out [b, s, H, d], stats)."""
    s = q.size(2)
    gamma0 = int(cfg.delta_lambda)
    window = int(cfg.sliding_window)
    sink = int(getattr(cfg, "sink", 1024))
    q_block = int(getattr(cfg, "q_block", 64))
    cut_n = s % gamma0 + max(128, gamma0)
    s_p = s - cut_n
    gamma_c = gamma0
    trigger = getattr(cfg, "stride_trigger", "absolute")
    history: List[float] = []
    parts, deltas, log = [], [], []
    for start, end in plan_chunks(s_p, int(cfg.adapt_chunk)):
        c_idx = torch.arange(start, end, gamma_c, device=q.device)
        delta = ops.anchor_deltas(q, k, v, c_idx, window=window, sink=sink, scaling=scaling, q_block=q_block)
        cos_mean, cos_min = interanchor_cos(delta)
        parts.append(c_idx)
        deltas.append(delta)
        log.append({"start": int(start), "gamma": int(gamma_c), "cos_mean": cos_mean, "cos_min": cos_min,
                    "n_anchors": int(c_idx.numel())})
        if trigger == "relative":
            gamma_c = next_gamma_relative(cos_mean, history, gamma_c, k=float(getattr(cfg, "adapt_k", 2.0)),
                                          gamma_min=int(cfg.gamma_min), gamma_max=int(cfg.gamma_max))
            history.append(cos_mean)
        else:
            gamma_c = next_gamma(cos_mean, gamma_c, threshold=float(cfg.adapt_threshold),
                                 gamma_min=int(cfg.gamma_min), gamma_max=int(cfg.gamma_max))
    idx = torch.cat(parts)
    # the chunks' anchor deltas are reused: the final call computes only the
    # dense tail rows and the windowed rows (delta_attention/llama.py:784-810)
    out = ops.prefill(q, k, v, gamma=gamma0, window=window, sink=sink, scaling=scaling, mode="delta",
                      q_block=q_block, anchors=idx, s_p=s_p, anchor_delta_in=torch.cat(deltas, dim=1))
    tail = torch.arange(s_p, s)
    stats: Dict[str, Any] = {
        "kind": "stride", "layer": int(layer_idx), "seq_len": int(s),
        "effective_sparsity": effective_sparsity(torch.cat((idx.cpu(), tail)), s, window, sink),
        "n_anchors": int(idx.numel()), "chunks": log,
    }
    return out, stats
