"""Shared helpers for the GPU parity tests (tolerances stated here)."""

import torch

# bf16 output tolerance (the reference uses 2e-2 max-abs for bf16 kernels,
# tests/test_math_identities.py:89; delta_kernel.py:376 uses atol 1e-2).
MAX_ABS = 1e-2
MIN_COS = 0.999


def cos_per_head(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Cosine over (rows, d) per head; inputs [b, n, H, d] -> [b, H]."""
    a = a.double().transpose(1, 2).reshape(a.shape[0], a.shape[2], -1)
    b = b.double().transpose(1, 2).reshape(b.shape[0], b.shape[2], -1)
    return torch.nn.functional.cosine_similarity(a, b, dim=-1)


def cos_per_row(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Cosine per (row, head) over d; [b, n, H, d] -> [b, n, H]."""
    return torch.nn.functional.cosine_similarity(a.double(), b.double(), dim=-1)


def assert_close(got: torch.Tensor, ref: torch.Tensor, what: str, max_abs: float = MAX_ABS,
                 min_cos: float = MIN_COS) -> None:
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - ref).abs().max().item()
    ch = cos_per_head(got, ref).min().item()
    cr = cos_per_row(got, ref)
    # per-row cosine is only meaningful for rows with non-negligible norm
    big = ref.norm(dim=-1) > 1e-3
    crm = cr[big].min().item() if big.any() else 1.0
    assert err <= max_abs, f"{what}: max abs err {err:.3e} > {max_abs}"
    assert ch >= min_cos, f"{what}: min per-head cos {ch:.6f} < {min_cos}"
    assert crm >= 0.99, f"{what}: min per-row cos {crm:.6f} < 0.99"
