"""Partitioning of delta-attention work over GPUs by KV-head group.

Every output row of query head h depends only on q-head h, its KV head and
its anchor, so a (sequence, KV group) pair -- a "unit" -- is independent of
every other unit: no collective runs inside attention.  A job of ``n_seqs``
sequences x ``n_kv_heads`` groups is dealt round-robin over ranks; a rank
stacks its units along the batch axis (q [n_units, G, N, d], k/v
[n_units, 1, N, d]) and runs one prefill over them.

``scaling="weak"``: the job has ``world`` sequences, so each rank owns
``n_kv_heads`` units whatever the world size.  ``scaling="strong"``: one
sequence, so each rank owns ``n_kv_heads / world`` groups.
"""

from __future__ import annotations

from typing import List, Tuple

Unit = Tuple[int, int]  # (sequence, kv group)


def job_units(n_seqs: int, n_kv_heads: int) -> List[Unit]:
    return [(s, g) for s in range(n_seqs) for g in range(n_kv_heads)]


def owned_units(n_seqs: int, n_kv_heads: int, world: int, rank: int) -> List[Unit]:
    """Units of this rank: unit index u = s * n_kv_heads + g goes to rank u % world."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return [u for i, u in enumerate(job_units(n_seqs, n_kv_heads)) if i % world == rank]


def job_for(scaling: str, world: int, n_kv_heads: int) -> int:
    """Number of sequences in the global job."""
    if scaling == "weak":
        return world
    if scaling == "strong":
        if n_kv_heads % world:
            raise ValueError(f"strong scaling needs world ({world}) to divide n_kv_heads ({n_kv_heads})")
        return 1
    raise ValueError(f"unknown scaling {scaling!r}")


def stack_units(q, k, v, units: List[Unit], group_size: int):
    """Gather this rank's units from full tensors q [S, H, N, d], k/v [S, Hkv, N, d]
    into the stacked per-rank layout."""
    import torch

    qs = torch.stack([q[s, g * group_size:(g + 1) * group_size] for s, g in units])
    ks = torch.stack([k[s, g:g + 1] for s, g in units])
    vs = torch.stack([v[s, g:g + 1] for s, g in units])
    return qs, ks, vs
