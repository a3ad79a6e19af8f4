"""The delta-attention plug-in surface, backed by the sm_100a kernels.

``DeltaAttention`` exposes the methods the reference's patched
``LlamaAttention`` dispatches to, with the same names, arguments, return
values and state:

* ``delta_forward``            <- ``delta_attention/llama.py:659-757``
* ``delta_adaptive_forward``   <- ``delta_attention/llama.py:759-824``
* ``sdpa_rectangle_forward``   <- ``delta_attention/llama.py:498-536``
* ``_decode_sparse_row``       <- ``delta_attention/llama.py:538-550``
* ``delta_decode_forward``     <- ``delta_attention/llama.py:552-634``

Inputs arrive post-projection and post-RoPE (``query_states`` [b, H, s, d],
``key_states``/``value_states`` [b, Hkv, n, d]); outputs are ``(attn_output
[b, s, H, d], None)``.  Knobs are read from ``self.config`` at call time, as
the reference does (``delta_attention/llama.py:673-675``).  RoPE-related
kwargs (``position_ids``, ``rope_sin``, ``rope_cos``) are accepted and ignored.

``register_attention_functions`` installs the same entry points under the
reference's attention-implementation names in transformers'
``AttentionInterface`` so an HF Llama/Qwen3 module (which carries
``.config``) can select them with ``attn_implementation``.
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import ops
from .drift import drift_summary


def _cfg(config, name, default):
    return getattr(config, name, default)


class DeltaAttention(torch.nn.Module):
    """Attention plug-in for one layer (holds the per-layer decode state)."""

    def __init__(self, config, layer_idx: int = 0):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        n_heads = int(config.num_attention_heads)
        n_kv = int(_cfg(config, "num_key_value_heads", n_heads))
        self.head_dim = int(_cfg(config, "head_dim", None) or config.hidden_size // n_heads)
        self.num_key_value_groups = n_heads // n_kv
        self.scaling = self.head_dim ** -0.5
        self._dec_state: Optional[Dict[str, Any]] = None
        self._dec_drift_points = None
        self._drift_stats = None
        self._stride_stats = None

    # ------------------------------------------------------------------
    # prefill
    # ------------------------------------------------------------------
    def delta_forward(self, module, query_states, key_states, value_states, attention_mask=None,
                      dropout: float = 0.0, scaling: float = 1.0, **kwargs) -> Tuple[torch.Tensor, None]:
        """Sparse (sink + block-anchored window) attention for every row, dense
        attention at every gamma-th row and the dense tail, delta broadcast --
        all inside the two kernel launches of ``ops.prefill``."""
        cfg = self.config
        gamma = int(cfg.delta_lambda)
        window = int(cfg.sliding_window)
        mode = _cfg(cfg, "mode", "delta")
        b, h, s, d = query_states.size()
        assert h == cfg.num_attention_heads, (h, s)
        if mode == "delta" and _cfg(cfg, "stride_policy", "fixed") == "adaptive":
            return self.delta_adaptive_forward(query_states, key_states, value_states, scaling), None
        log_drift = bool(_cfg(cfg, "log_drift", False)) and mode == "delta"
        res = ops.prefill(query_states, key_states, value_states, gamma=gamma, window=window,
                          sink=int(_cfg(cfg, "sink", 1024)), scaling=scaling, mode=mode,
                          q_block=int(_cfg(cfg, "q_block", 64)), return_anchor_delta=log_drift)
        if log_drift:
            out, delta = res
            if delta.size(1) >= 2:
                self._drift_stats = drift_summary(delta, self.layer_idx, gamma, s)
            return out, None
        return res, None

    def delta_adaptive_forward(self, query_states, key_states, value_states, scaling):
        """Chunked adaptive anchor placement (``delta_attention/llama.py:759-824``)."""
        from .stride import adaptive_prefill

        out, stats = adaptive_prefill(self.config, query_states, key_states, value_states, scaling,
                                      layer_idx=self.layer_idx)
        self._stride_stats = stats
        return out

    # ------------------------------------------------------------------
    # decode
    # ------------------------------------------------------------------
    def sdpa_rectangle_forward(self, module, query_states, key_states, value_states, attention_mask=None,
                               dropout: float = 0.0, scaling: float = 1.0, **kwargs):
        """Dense attention of ``s`` new rows over ``n`` cached keys with the
        rectangle mask ``tril(n - s)``; single-token steps go to the
        sparse/delta decode path when ``decode_mode != "dense"``."""
        b, _, s, d = query_states.size()
        if s == 1 and _cfg(self.config, "decode_mode", "dense") != "dense":
            return self.delta_decode_forward(module, query_states, key_states, value_states, scaling=scaling)
        n = key_states.size(2)
        if s == 1:
            dense, _ = ops.decode(query_states, key_states, value_states, window=0, sink=0, scaling=scaling,
                                  want_dense=True, want_sparse=False)
            return dense, None
        rows = torch.arange(s, device=query_states.device, dtype=torch.int32)
        out = ops.rows(query_states, key_states, value_states, rows, rows + (n - s), scaling=scaling,
                       validate=False)
        return out, None

    def _decode_sparse_row(self, q, k, v, scaling):
        """StreamingLLM decode row: the first ``sink`` keys plus the last
        ``sliding_window`` keys (all keys when the cache is shorter).
        Returns [b, 1, H, d]."""
        _, sparse = ops.decode(q, k, v, window=int(self.config.sliding_window),
                               sink=int(_cfg(self.config, "sink", 1024)), scaling=scaling,
                               want_dense=False, want_sparse=True)
        return sparse

    def delta_decode_forward(self, module, query_states, key_states, value_states, scaling=1.0, **kwargs):
        """Sparse decode with a cached, periodically refreshed delta.

        Per-layer state ``_dec_state = {last_delta, steps, last_sparse, cos_hist}``.
        Anchor when: no delta yet | steps+1 >= gamma_dec_max | fixed policy and
        steps+1 >= gamma_dec | drift policy cos < drift_threshold | drift_rel
        cos < mean - drift_k*std of the last 16 (>= 8 entries).  Anchors output
        the dense row and refresh the delta; other steps output sparse + delta.
        When the anchor decision is known before attention runs (first step,
        cap, fixed policy), the dense and sparse rows come from ONE pass over
        the cache.  Batch > 1 shares one schedule per layer.
        """
        cfg = self.config
        mode = cfg.decode_mode
        assert mode in ("sparse", "delta"), mode
        q, k, v = query_states, key_states, value_states
        window = int(cfg.sliding_window)
        sink = int(_cfg(cfg, "sink", 1024))
        if mode == "sparse":
            return self._decode_sparse_row(q, k, v, scaling), None

        st = self._dec_state or {"last_delta": None, "steps": 0, "last_sparse": None, "cos_hist": []}
        log_drift = bool(_cfg(cfg, "log_drift", False))
        policy = _cfg(cfg, "refresh_policy", "fixed")

        def _cos(a, b):
            return torch.nn.functional.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0).item()

        # decide as much as possible before touching the cache
        if st["last_delta"] is None:
            anchor, cur, decided = True, 0, True
        else:
            cur = st["steps"] + 1
            anchor = cur >= int(_cfg(cfg, "gamma_dec_max", 128))
            if policy == "fixed" and cur >= int(cfg.gamma_dec):
                anchor = True
            decided = anchor or policy not in ("drift", "drift_rel") or st["last_sparse"] is None
        want_dense_now = (decided and anchor) or log_drift
        dense_out, sparse_out = ops.decode(q, k, v, window=window, sink=sink, scaling=scaling,
                                           want_dense=want_dense_now, want_sparse=True)
        if not decided:
            c = _cos(sparse_out, st["last_sparse"])
            if policy == "drift":
                anchor = c < float(cfg.drift_threshold)
            else:
                hist = st["cos_hist"]
                if len(hist) >= 8:
                    mu = sum(hist) / len(hist)
                    sd = (sum((x - mu) ** 2 for x in hist) / len(hist)) ** 0.5
                    anchor = c < mu - float(_cfg(cfg, "drift_k", 2.0)) * sd
                hist.append(c)
                del hist[:-16]
            if anchor and dense_out is None:
                dense_out, _ = ops.decode(q, k, v, window=window, sink=sink, scaling=scaling,
                                          want_dense=True, want_sparse=False)
        if anchor:
            st["last_delta"] = dense_out - sparse_out
            st["steps"] = 0
            out = dense_out
        else:
            out = sparse_out + st["last_delta"]
            st["steps"] = cur
        if log_drift:
            true_delta = dense_out - sparse_out
            pts = self._dec_drift_points or []
            pts.append({"steps_since_anchor": int(cur), "anchor": bool(anchor),
                        "drift_cos": _cos(true_delta, st["last_delta"]),
                        "applied_vs_true_cos": _cos(out, dense_out)})
            self._dec_drift_points = pts
        st["last_sparse"] = sparse_out
        self._dec_state = st
        return out, None

    def check(self) -> None:
        """Raise ``DtaError`` if a kernel launched on this layer's device since
        the last check gave up on a bounded wait or met an out-of-range row
        (synchronises the current stream; see ``ops.check_errors``)."""
        ops.check_errors()

    def reset_decode_state(self) -> None:
        """Called at every new prefill (``delta_attention/sample.py:148-151``)."""
        self._dec_state = None
        self._dec_drift_points = None


# ----------------------------------------------------------------------
# transformers AttentionInterface registration
# ----------------------------------------------------------------------
def _plugin(module) -> DeltaAttention:
    p = getattr(module, "_delta_plugin", None)
    if p is None:
        p = DeltaAttention(module.config, layer_idx=int(getattr(module, "layer_idx", 0) or 0))
        module._delta_plugin = p
    p.config = module.config
    return p


def window_attention(module, query, key, value, attention_mask=None, scaling=None, dropout=0.0, **kwargs):
    """``attn_implementation="window"``: prefill through ``delta_forward``,
    single-token steps through ``sdpa_rectangle_forward``."""
    p = _plugin(module)
    scaling = p.scaling if scaling is None else scaling
    if query.size(2) == 1 and key.size(2) > 1:
        return p.sdpa_rectangle_forward(module, query, key, value, attention_mask, dropout, scaling, **kwargs)
    if key.size(2) != query.size(2):
        return p.sdpa_rectangle_forward(module, query, key, value, attention_mask, dropout, scaling, **kwargs)
    p.reset_decode_state()
    return p.delta_forward(module, query, key, value, attention_mask, dropout, scaling, **kwargs)


def sdpa_rectangle_attention(module, query, key, value, attention_mask=None, scaling=None, dropout=0.0, **kwargs):
    p = _plugin(module)
    scaling = p.scaling if scaling is None else scaling
    return p.sdpa_rectangle_forward(module, query, key, value, attention_mask, dropout, scaling, **kwargs)


def register_attention_functions() -> bool:
    """Register ``window``/``hip_attention``/``sdpa_rectangle`` in transformers'
    attention registry (``delta_attention/sample.py:266-268``).  Returns False
    when transformers is unavailable."""
    try:
        from transformers import AttentionInterface
    except Exception:  # pragma: no cover - transformers missing
        return False
    AttentionInterface.register("window", window_attention)
    AttentionInterface.register("hip_attention", window_attention)
    AttentionInterface.register("sdpa_rectangle", sdpa_rectangle_attention)
    return True
