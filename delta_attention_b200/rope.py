"""Rotary position embedding used to build post-RoPE q/k inputs.

The delta plug-in receives q/k AFTER RoPE (``delta_attention/llama.py:845-862``),
so RoPE is upstream of every kernel in this package.  It is provided here so
synthetic inputs (``synthetic.make_inputs``) and the random-init models carry
the same rotary structure as the reference's Llama/Qwen3 attention:
``rotate_half`` / ``apply_rotary_pos_emb`` (``delta_attention/llama.py:161-192``)
with the default and the ``llama3`` frequency schedules
(``LlamaRotaryEmbedding``, ``delta_attention/llama.py:83-158``; the llama3
schedule is the one published with Llama 3.1: wavelengths above
``old_ctx / low_freq_factor`` are divided by ``factor``, those below
``old_ctx / high_freq_factor`` are kept, and the band between is blended
linearly in ``old_ctx / wavelength``).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch


def inv_freq(head_dim: int, theta: float, llama3: Optional[dict] = None,
             device=None) -> torch.Tensor:
    """Inverse frequencies ``theta ** (-2i/d)`` (float32), optionally with the
    llama3 long-context schedule ``{"factor", "low_freq_factor",
    "high_freq_factor", "original_max_position_embeddings"}``."""
    f = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64, device=device) / head_dim))
    if llama3:
        factor = float(llama3.get("factor", 8.0))
        lo = float(llama3.get("low_freq_factor", 1.0))
        hi = float(llama3.get("high_freq_factor", 4.0))
        old = float(llama3.get("original_max_position_embeddings", 8192))
        wavelen = 2 * math.pi / f
        smooth = (old / wavelen - lo) / (hi - lo)
        scaled = torch.where(wavelen > old / lo, f / factor, f)
        mid = (1 - smooth) * f / factor + smooth * f
        is_mid = (wavelen <= old / lo) & (wavelen >= old / hi)
        f = torch.where(is_mid, mid, scaled)
    return f.to(torch.float32)


def cos_sin(positions: torch.Tensor, head_dim: int, theta: float,
            llama3: Optional[dict] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [n, head_dim] (``emb = cat(freqs, freqs)``)."""
    f = inv_freq(head_dim, theta, llama3, device=positions.device)
    freqs = positions.to(torch.float32)[:, None] * f[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x * cos + rotate_half(x) * sin`` with cos/sin broadcast over the
    sequence axis (dim -2) of ``x`` [..., s, d]."""
    return x * cos + rotate_half(x) * sin
