"""Host-side multi-GPU logic on CPU: KV-group unit assignment across ranks and
the max-over-ranks timing reduction, with world_size-2 gloo process groups."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from delta_attention_b200.sharding import job_for, job_units, owned_units, stack_units


def test_units_cover_job_disjointly():
    for world in (1, 2, 4, 8):
        for scaling in ("weak", "strong"):
            n_seqs = job_for(scaling, world, 8)
            owned = [owned_units(n_seqs, 8, world, r) for r in range(world)]
            flat = [u for o in owned for u in o]
            assert sorted(flat) == sorted(job_units(n_seqs, 8))
            sizes = {len(o) for o in owned}
            assert sizes == ({8} if scaling == "weak" else {8 // world})


def test_stack_units_layout():
    S, H, Hkv, N, d = 2, 8, 2, 16, 4
    q = torch.randn(S, H, N, d)
    k = torch.randn(S, Hkv, N, d)
    units = owned_units(S, Hkv, 2, 1)
    qs, ks, vs = stack_units(q, k, k, units, H // Hkv)
    for i, (s, g) in enumerate(units):
        assert torch.equal(qs[i], q[s, 4 * g:4 * g + 4])
        assert torch.equal(ks[i, 0], k[s, g])


def _worker(rank, world, port, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    units = owned_units(job_for("weak", world, 8), 8, world, rank)
    gathered = [None] * world
    dist.all_gather_object(gathered, units)
    t = torch.tensor([10.0 + rank], dtype=torch.float64)  # this rank's elapsed ms
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        ret.put((gathered, t.item()))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_assignment_and_max_timing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat = [tuple(u) for g in gathered for u in g]
    assert sorted(flat) == job_units(2, 8)
    assert tmax == 11.0
