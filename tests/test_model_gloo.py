"""The tensor-parallel decoder on CPU (no GPU): its KV-cache decode path must
reproduce a full forward pass, and world-size-2 tensor parallelism over gloo
must reproduce the single-rank model.  Attention is replaced by a dense causal
torch attention here (the plug-in's kernels need a B200; the GPU tests run
the model through them)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from delta_attention_b200.config import Config
from delta_attention_b200.model import LLAMA31_8B, QWEN3_8B, TP, DeltaDecoder, tiny

TINY = dict(n_layers=2, hidden=256, n_heads=8, n_kv_heads=2, head_dim=32, intermediate=512, vocab=1000)


def dense_causal(i, q, k, v, scaling, prefill):
    """q [B,H,s,d], k/v [B,Hkv,n,d]: row j (position n-s+j) sees keys <= its position."""
    B, H, s, d = q.shape
    n, G = k.shape[2], H // k.shape[1]
    k = k.repeat_interleave(G, dim=1).float()
    v = v.repeat_interleave(G, dim=1).float()
    pos = torch.arange(n - s, n)[:, None]
    mask = torch.arange(n)[None, :] <= pos
    o = torch.nn.functional.scaled_dot_product_attention(q.float(), k, v, attn_mask=mask, scale=scaling)
    return o.transpose(1, 2).to(q.dtype)


def _model(arch, tp=None, seed=3):
    return DeltaDecoder(tiny(arch, **TINY), Config(), tp=tp, device="cpu", dtype=torch.float32, seed=seed,
                        attention=dense_causal, init_std=0.05)


@pytest.mark.parametrize("arch", [LLAMA31_8B, QWEN3_8B], ids=["llama", "qwen3"])
def test_cached_decode_matches_full_forward(arch):
    ids = torch.randint(0, TINY["vocab"], (2, 20), generator=torch.Generator().manual_seed(0))
    full = _model(arch)
    full.allocate_cache(2, 32)
    x_full = full.forward(ids)
    step = _model(arch)
    step.allocate_cache(2, 32)
    outs = [step.forward(ids[:, :16])]
    for j in range(16, 20):  # the decode path: one position at a time over the cache
        outs.append(step.forward(ids[:, j:j + 1]))
    torch.testing.assert_close(torch.cat(outs, dim=1), x_full, rtol=1e-4, atol=1e-4)
    assert step.length == 20


def test_prefill_then_greedy_tokens():
    m = _model(LLAMA31_8B)
    m.allocate_cache(1, 24)
    ids = torch.randint(0, TINY["vocab"], (1, 12), generator=torch.Generator().manual_seed(1))
    tok = m.prefill(ids)
    seq = [tok]
    for _ in range(3):
        seq.append(m.decode_step(seq[-1]))
    assert m.length == 15 and all(0 <= int(t) < TINY["vocab"] for t in seq)
    # the first token is the argmax of the prefill logits
    m2 = _model(LLAMA31_8B)
    m2.allocate_cache(1, 24)
    logits = m2.logits_last(m2.forward(ids)[:, -1])
    assert int(logits.argmax(-1)) == int(tok)


def _tp_worker(rank, world, port, arch_name, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    arch = {"llama": LLAMA31_8B, "qwen3": QWEN3_8B}[arch_name]
    ids = torch.randint(0, TINY["vocab"], (2, 12), generator=torch.Generator().manual_seed(2))
    m = _model(arch, tp=TP(rank, world, None))
    m.allocate_cache(2, 16)
    logits = m.logits_last(m.forward(ids)[:, -1])
    step = m.logits_last(m.forward(ids[:, :1] * 0 + 7)[:, -1])  # one cached decode position
    if rank == 0:
        # numpy arrays travel by value (a torch tensor would pass a shared-memory
        # handle that must outlive this process until the parent has opened it)
        ret.put((logits.detach().numpy().copy(), step.detach().numpy().copy()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("arch_name", ["llama", "qwen3"])
def test_two_rank_tensor_parallel_matches_one_rank(arch_name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300 + (0 if arch_name == "llama" else 1)
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, arch_name, q)) for r in range(2)]
    for p in procs:
        p.start()
    logits_tp, step_tp = (torch.from_numpy(a) for a in q.get(timeout=180))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    arch = {"llama": LLAMA31_8B, "qwen3": QWEN3_8B}[arch_name]
    ids = torch.randint(0, TINY["vocab"], (2, 12), generator=torch.Generator().manual_seed(2))
    m = _model(arch)
    m.allocate_cache(2, 16)
    logits = m.logits_last(m.forward(ids)[:, -1])
    step = m.logits_last(m.forward(ids[:, :1] * 0 + 7)[:, -1])
    torch.testing.assert_close(logits_tp, logits, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(step_tp, step, rtol=1e-4, atol=1e-4)
