"""End-to-end model benchmark: TTFT and decode tokens/s of the tensor-parallel
decoder (BASELINE configs 3 and 4), one process per GPU.

    # config 3: Llama-3.1-8B, one 131072-token prompt, 128 dense decode tokens
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m delta_attention_b200.model_bench --arch llama
    # config 4: Qwen3-8B, 4 x 65536-token prompts, 256 delta-mode decode tokens
    python -m torch.distributed.run ... -m delta_attention_b200.model_bench \\
        --arch qwen3 --batch 4 --seq 65536 --new-tokens 256 --decode-mode delta

Weights are random (bf16, seeded) and the prompt is uniform-random token ids:
no checkpoint or dataset is involved.  Times are CUDA-event times on each
rank, maximum over ranks.  Rank 0 prints one JSON line with the TTFT (prefill
of the prompt and the first token), prefill and decode tokens/s, and a
breakdown of the prefill and of a few extra decode steps into attention (the
plug-in's kernels), GEMMs with their elementwise work, and the all-reduces of
the row-parallel projections (the collective that limits multi-GPU scaling).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--arch", choices=["llama", "qwen3"], default="llama")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--new-tokens", type=int, default=128)
    ap.add_argument("--decode-mode", choices=["dense", "sparse", "delta"], default="dense")
    ap.add_argument("--window", type=int, default=2048)
    ap.add_argument("--sink", type=int, default=128)
    ap.add_argument("--gamma", type=int, default=64)
    ap.add_argument("--gamma-dec", type=int, default=32)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (0 = the architecture's)")
    ap.add_argument("--breakdown-steps", type=int, default=8)
    ap.add_argument("--eager-decode", action="store_true",
                    help="decode through the eager path (one launch sequence per layer from Python) "
                         "instead of one CUDA-graph replay per token")
    return ap.parse_args(argv)


def _max_over_ranks(vals, world, dev):
    if world == 1:
        return vals
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def _phase_ms(events):
    return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in events.items()}


def main(argv=None) -> int:
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from . import ops
    from .config import Config
    from .model import ARCHS, TP, DecodeGraph, DeltaDecoder, tiny

    arch = ARCHS[args.arch]
    if args.layers:
        arch = tiny(arch, n_layers=args.layers)
    cfg = Config(delta_lambda=args.gamma, sliding_window=args.window, sink=args.sink, mode="delta",
                 decode_mode=args.decode_mode, gamma_dec=args.gamma_dec)
    model = DeltaDecoder(arch, cfg, TP(rank, world), device=dev, seed=0)
    g = torch.Generator(device=dev).manual_seed(1234)
    ids = torch.randint(0, arch.vocab, (args.batch, args.seq), generator=g, device=dev)
    model.allocate_cache(args.batch, args.seq + args.new_tokens + args.breakdown_steps + 1)

    # warm-up: a short prompt and a few steps (kernels, cuBLAS heuristics, NCCL;
    # the decode graphs are captured here)
    graph = None if args.eager_decode else DecodeGraph(model, args.batch)
    warm = ids[:, :min(args.seq, 8192)]
    tok = model.prefill(warm)
    if graph is not None:
        graph.start(tok)
    for _ in range(3):
        tok = graph.step() if graph is not None else model.decode_step(tok)
    torch.cuda.synchronize()
    ops.check_errors()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    # TTFT: prefill of the whole prompt and the first token
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    tok = model.prefill(ids)
    e1.record()
    torch.cuda.synchronize()
    ttft = e0.elapsed_time(e1)
    # decode
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    if graph is not None:
        graph.start(tok)
        for _ in range(args.new_tokens):
            graph.step()
        tok = graph.tok.clone()
    else:
        for _ in range(args.new_tokens):
            tok = model.decode_step(tok)
    d1.record()
    torch.cuda.synchronize()
    dec_ms = d0.elapsed_time(d1)
    ops.check_errors()
    # breakdowns (separate runs with CUDA events around each phase of every layer)
    model.events = {}
    barrier()
    model.prefill(ids[:, :args.seq])
    torch.cuda.synchronize()
    pre_phase = _phase_ms(model.events)
    model.events = {}
    for _ in range(args.breakdown_steps):
        tok = model.decode_step(tok)
    torch.cuda.synchronize()
    dec_phase = {k: v / max(1, args.breakdown_steps) for k, v in _phase_ms(model.events).items()}
    model.events = None
    ops.check_errors()

    keys = ("attention", "gemm", "all_reduce")
    vals = [ttft, dec_ms] + [pre_phase.get(k, 0.0) for k in keys] + [dec_phase.get(k, 0.0) for k in keys]
    vals = _max_over_ranks(vals, world, dev)
    ttft, dec_ms = vals[0], vals[1]
    pre = dict(zip(keys, vals[2:5]))
    dec = dict(zip(keys, vals[5:8]))
    if rank == 0:
        layer_bytes = args.batch * args.seq * arch.hidden * 2
        line = {
            "workload": ("config3" if args.arch == "llama" else "config4") + f": {arch.name}, random-init bf16, "
                        f"TP over KV groups, delta prefill, {args.decode_mode} decode",
            "arch": arch.name, "n_layers": arch.n_layers, "n_gpus": world, "batch": args.batch,
            "prompt_tokens": args.seq, "new_tokens": args.new_tokens, "decode_mode": args.decode_mode,
            "window": args.window, "sink": args.sink, "gamma": args.gamma,
            "ttft_ms": ttft,
            "prefill_tokens_per_s": args.batch * args.seq / (ttft / 1e3),
            "decode_path": "eager" if args.eager_decode else "cuda graph per token",
            "decode_ms_per_step": dec_ms / args.new_tokens,
            "decode_tokens_per_s": args.batch * args.new_tokens / (dec_ms / 1e3),
            "prefill_breakdown_ms": pre, "decode_breakdown_ms_per_step": dec,
            "all_reduces_per_layer": 2 if world > 1 else 0,
            "prefill_all_reduce_bytes": layer_bytes if world > 1 else 0,
            "data": "synthetic (uniform-random token ids, seeded random-init weights)",
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        graph.release()  # graphs holding NCCL work go before the process group
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
