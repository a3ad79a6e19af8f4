"""Anchor-delta drift telemetry (``delta_attention/drift.py``).

``drift_summary`` consumes the per-anchor deltas the prefill kernel emits
(``ops.prefill(..., return_anchor_delta=True)``) instead of materialising
them with torch ops; the summary format and histogram constants are the
reference's (``delta_attention/drift.py:17-49``) so sidecar files aggregate
with the reference's own tooling.
"""

from __future__ import annotations

from typing import Any, Dict

HIST_BINS = 40
HIST_RANGE = (-1.0, 1.0)


def drift_summary(dense_sparse_diff, layer_idx: int, gamma: int, seq_len: int) -> Dict[str, Any]:
    """Per-layer summary of cos(delta_i, delta_{i+1}) over consecutive anchors, per head.
    ``dense_sparse_diff``: [b, n_anchors, h, d]."""
    import torch

    a = dense_sparse_diff[:, :-1].float()
    b = dense_sparse_diff[:, 1:].float()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=-1)
    flat = cos.flatten()
    hist = torch.histc(flat, bins=HIST_BINS, min=HIST_RANGE[0], max=HIST_RANGE[1])
    q = torch.quantile(flat, torch.tensor([0.1, 0.5, 0.9], device=flat.device))
    return {
        "layer": int(layer_idx), "gamma": int(gamma), "seq_len": int(seq_len), "n": int(flat.numel()),
        "mean": float(flat.mean().item()), "p10": float(q[0].item()), "p50": float(q[1].item()),
        "p90": float(q[2].item()), "hist_bins": HIST_BINS, "hist_range": list(HIST_RANGE),
        "hist": [int(x) for x in hist.tolist()],
    }
