"""Seeded synthetic q/k/v in the shapes the delta plug-in receives.

No public dataset is involved in the reference's headline measurement
(``eval/anchor_bench.py:145-165`` draws random q/k/v); the recipe here is
i.i.d. ``N(0, 1) * std`` from a seeded ``torch.Generator`` (the draw order of
``delta_attention/validation.py:133-145``: q, then k, then v) followed by RoPE
on q and k.  Inputs are produced in float32 and rounded to the compute dtype,
so CPU checkers can be fed exactly the values the GPU sees.
"""

from __future__ import annotations

import hashlib
from typing import Optional, Tuple

import torch

from .rope import apply_rope, cos_sin


def make_inputs(s: int, n_heads: int = 32, n_kv_heads: int = 8, head_dim: int = 128,
                seed: int = 0, std: float = 0.5, rope_theta: Optional[float] = 500000.0,
                dtype: torch.dtype = torch.bfloat16, device="cpu", batch: int = 1,
                gen_device: str = "cpu") -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """q [b, H, s, d], k/v [b, Hkv, s, d] (contiguous), post-RoPE, in ``dtype``.

    ``gen_device="cuda"`` draws on the GPU (fast at 128K tokens); CPU draws are
    the reproducible default for tests.
    """
    gen = torch.Generator(device=gen_device).manual_seed(seed)
    kw = dict(generator=gen, dtype=torch.float32, device=gen_device)
    q = torch.randn(batch, n_heads, s, head_dim, **kw) * std
    k = torch.randn(batch, n_kv_heads, s, head_dim, **kw) * std
    v = torch.randn(batch, n_kv_heads, s, head_dim, **kw) * std
    if rope_theta:
        cos, sin = cos_sin(torch.arange(s, device=gen_device), head_dim, rope_theta)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
    return (q.to(device=device, dtype=dtype), k.to(device=device, dtype=dtype),
            v.to(device=device, dtype=dtype))


def tensor_digest(*tensors: torch.Tensor) -> str:
    """sha256 over the raw bytes of the given tensors (CPU copies)."""
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().contiguous().cpu()
        h.update(t.view(torch.uint8).reshape(-1).numpy().tobytes() if t.dtype == torch.bfloat16
                 else t.numpy().tobytes())
    return h.hexdigest()
