"""Generate golden fixtures from the reference implementation (run on CPU).

Usage (needs the reference checkout; writes ``tests/golden/*.npz|json``)::

    python tests/golden/make_golden.py --reference /path/to/delta-attention

What is run, all from the reference's own source:

* ``delta_attention/train/flex_delta.py`` ``delta_forward_train`` -- the
  reference's CPU-runnable restatement of the prefill path.  Two module
  attributes are patched from outside so it runs eagerly on CPU:
  ``_flex`` is set to the eager ``flex_attention`` and the module's
  ``create_block_mask`` is wrapped to force ``_compile=False`` (the compiled
  variants need a GPU / a working inductor toolchain).
* ``delta_attention/stride.py`` ``apply_delta_variable`` and
  ``uniform_effective_sparsity``; ``delta_attention/validation.py``
  ``anchor_indices``.
* the decode methods ``repeat_kv``, ``_decode_sparse_row`` and
  ``delta_decode_forward`` of ``delta_attention/llama.py``.  That module cannot
  be imported here (it needs transformers 4.51 and hip-attn), so the three
  function definitions are located in the file with ``ast`` and executed in a
  namespace that provides ``torch`` and SDPA; they run on a stand-in ``self``
  carrying the config fields they read.

Inputs are regenerated deterministically by
``delta_attention_b200.synthetic.make_inputs``; each fixture records the
sha256 of its bf16 inputs so a drift in the generator is detected.  The
reference runs in float32 on the bf16-rounded inputs (the values the CUDA
kernels consume).
"""

from __future__ import annotations

import argparse
import ast
import functools
import json
import os
import sys
import time
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from delta_attention_b200.synthetic import make_inputs, tensor_digest  # noqa: E402

# name: (s, H, Hkv, d, gamma, window, sink, rope_theta, seed, sample_rows or None=full)
FLEX_CASES = {
    "flex_small_gqa4": (512, 4, 1, 64, 64, 128, 32, 500000.0, 0, None),
    "flex_g16_d128": (1024, 4, 1, 128, 16, 256, 64, 500000.0, 1, 96),
    "flex_gamma1": (512, 4, 2, 64, 1, 128, 32, None, 2, 96),
    "flex_fullwindow": (512, 4, 1, 64, 64, 512, 32, 500000.0, 3, 96),
    "flex_gqa8_g128": (1024, 8, 1, 128, 128, 256, 128, 500000.0, 4, 96),
    "flex_g32_w64": (768, 4, 2, 64, 32, 64, 16, 10000.0, 5, 96),
    # config 1 of the benchmark matrix (CPU-runnable reference case)
    "flex_config1": (4096, 32, 8, 128, 64, 1024, 64, 500000.0, 0, 64),
}


def _sample_rows(s: int, gamma: int, n: int, seed: int) -> torch.Tensor:
    cut_n = s % gamma + max(128, gamma)
    s_p = s - cut_n
    g = torch.Generator().manual_seed(1000 + seed)
    rnd = torch.randperm(s, generator=g)[: n // 2]
    anchors = torch.arange(0, max(s_p, 0), gamma)
    a = anchors[torch.randperm(anchors.numel(), generator=g)[: n // 8]] if anchors.numel() else anchors
    tail = torch.arange(max(s_p, 0), s)
    t = tail[torch.randperm(tail.numel(), generator=g)[: n // 8]]
    ends = torch.tensor([0, s - 1, max(s_p - 1, 0), max(s_p, 0) % s])
    return torch.unique(torch.cat((rnd, a, t, ends)))


def load_flex(ref: str):
    sys.path.insert(0, ref)
    from delta_attention.train import flex_delta
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention

    flex_delta._flex = flex_attention
    orig = create_block_mask

    @functools.wraps(orig)
    def _eager_block_mask(*a, **kw):
        kw["_compile"] = False
        return orig(*a, **kw)

    flex_delta.create_block_mask = _eager_block_mask
    flex_delta.get_block_mask.cache_clear()
    return flex_delta


def gen_flex(ref: str, out_dir: str, only=None) -> None:
    flex_delta = load_flex(ref)
    torch.set_num_threads(os.cpu_count() or 1)
    for name, (s, H, Hkv, d, gamma, window, sink, theta, seed, nsamp) in FLEX_CASES.items():
        if only and name not in only:
            continue
        q, k, v = make_inputs(s, H, Hkv, d, seed=seed, rope_theta=theta, dtype=torch.bfloat16)
        digest = tensor_digest(q, k, v)
        t0 = time.time()
        with torch.no_grad():
            out = flex_delta.delta_forward_train(q.float(), k.float(), v.float(), gamma=gamma,
                                                 window=window, sink=sink)  # [1, s, H, d]
        dt = time.time() - t0
        rec = dict(s=s, H=H, Hkv=Hkv, d=d, gamma=gamma, window=window, sink=sink,
                   rope_theta=-1.0 if theta is None else theta, seed=seed, digest=digest)
        arrays = {"checksum": out[0].double().sum(dim=0).numpy()}  # [H, d]
        if nsamp is None:
            arrays["rows"] = np.arange(s)
            arrays["out"] = out[0].float().numpy()
        else:
            rows = _sample_rows(s, gamma, nsamp, seed)
            arrays["rows"] = rows.numpy()
            arrays["out"] = out[0, rows].float().numpy()
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), meta=json.dumps(rec), **arrays)
        print(f"[golden] {name}: s={s} H={H}/{Hkv} d={d} gamma={gamma} W={window} S={sink} "
              f"-> {arrays['out'].shape} in {dt:.1f}s", flush=True)


def gen_stride(ref: str, out_dir: str) -> None:
    sys.path.insert(0, ref)
    from delta_attention import stride, validation

    g = torch.Generator().manual_seed(7)
    s_p, n_h, d = 300, 3, 16
    sparse = torch.randn(1, s_p, n_h, d, generator=g)
    idx = torch.tensor([0, 5, 17, 40, 41, 100, 180, 256, 299])
    dense_sel = torch.randn(1, idx.numel(), n_h, d, generator=g)
    corrected = stride.apply_delta_variable(sparse, dense_sel, idx, s_p)
    layouts = []
    for s_, gm in [(4096, 64), (131072, 64), (32768, 16), (65536, 32), (131072, 128), (1000, 8),
                   (8192, 1), (5000, 256), (130, 1)]:
        a, t = validation.anchor_indices(s_, gm)
        layouts.append(dict(s=s_, gamma=gm, n_anchor=int(a.numel()), n_tail=int(t.numel()),
                            first_tail=int(t[0]) if t.numel() else -1,
                            anchor_sum=int(a.sum()),
                            eff=stride.uniform_effective_sparsity(s_, gm, 2048, 128)))
    gam = []
    for cm, gc in [(0.5, 64), (0.96, 64), (0.99, 64), (0.99, 256), (0.1, 16)]:
        gam.append(dict(cos=cm, gamma=gc, nxt=stride.next_gamma(cm, gc, threshold=0.95, gamma_min=16,
                                                                 gamma_max=256)))
    rel = []
    hist = [0.6, 0.62, 0.58, 0.61]
    for cm, gc in [(0.3, 64), (0.9, 64), (0.6, 64)]:
        rel.append(dict(cos=cm, gamma=gc, nxt=stride.next_gamma_relative(cm, hist, gc, k=2.0, gamma_min=16,
                                                                          gamma_max=256)))
    np.savez_compressed(os.path.join(out_dir, "stride_variable.npz"), sparse=sparse.numpy(),
                        idx=idx.numpy(), dense_sel=dense_sel.numpy(), corrected=corrected.numpy(),
                        meta=json.dumps(dict(s_p=s_p, layouts=layouts, next_gamma=gam,
                                             next_gamma_relative=rel, hist=hist)))
    print("[golden] stride_variable", flush=True)


def _load_llama_functions(ref: str):
    """Execute ``repeat_kv`` and the two decode methods from the reference's
    llama.py source in an isolated namespace."""
    path = os.path.join(ref, "delta_attention", "llama.py")
    src = open(path, encoding="utf-8").read()
    tree = ast.parse(src)
    wanted = {"repeat_kv": None, "_decode_sparse_row": None, "delta_decode_forward": None}
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name in wanted and wanted[node.name] is None:
            wanted[node.name] = ast.get_source_segment(src, node)
    import textwrap

    ns = {"torch": torch, "sdpa": torch.nn.functional.scaled_dot_product_attention}
    for name, code in wanted.items():
        exec(compile(textwrap.dedent(code), path, "exec"), ns)  # noqa: S102
    return ns


DECODE_SHAPE = dict(n_keys=2000, window=512, steps=14, seed=11)


def decode_inputs():
    """Decode-step inputs (bf16-rounded, held in float32): 14 query rows
    [1,32,1,64] and one KV cache [1,8,2000,64] (> sink 1024 + window 512)."""
    g = torch.Generator().manual_seed(DECODE_SHAPE["seed"])
    qs = [torch.randn(1, 32, 1, 64, generator=g).to(torch.bfloat16).float()
          for _ in range(DECODE_SHAPE["steps"])]
    k = torch.randn(1, 8, DECODE_SHAPE["n_keys"], 64, generator=g).to(torch.bfloat16).float()
    v = torch.randn(1, 8, DECODE_SHAPE["n_keys"], 64, generator=g).to(torch.bfloat16).float()
    return qs, k, v


def gen_decode(ref: str, out_dir: str) -> None:
    ns = _load_llama_functions(ref)

    class _Cfg:
        pass

    def make_self(**cfg):
        self = types.SimpleNamespace()
        self.config = _Cfg()
        for k_, v_ in cfg.items():
            setattr(self.config, k_, v_)
        self.num_key_value_groups = 4
        self.layer_idx = 0
        self._dec_state = None
        self._decode_sparse_row = types.MethodType(ns["_decode_sparse_row"], self)
        return self

    rec = {}
    arrays = {}
    n_keys, window, steps = DECODE_SHAPE["n_keys"], DECODE_SHAPE["window"], DECODE_SHAPE["steps"]
    qs, k, v = decode_inputs()
    rec["digest"] = tensor_digest(torch.stack(qs), k, v)
    scaling = 64 ** -0.5
    for policy, extra in [("fixed", dict(gamma_dec=3)), ("drift", dict(gamma_dec=32, drift_threshold=0.5)),
                          ("drift_rel", dict(gamma_dec=32, drift_k=0.25))]:
        self = make_self(decode_mode="delta", sliding_window=window, refresh_policy=policy,
                         gamma_dec_max=128, log_drift=False, drift_threshold=extra.get("drift_threshold", 0.95),
                         drift_k=extra.get("drift_k", 2.0), gamma_dec=extra["gamma_dec"])
        outs, flags = [], []
        for t in range(steps):
            out, _ = ns["delta_decode_forward"](self, self, qs[t], k, v, scaling=scaling)
            outs.append(out)
            flags.append(bool(self._dec_state["steps"] == 0))
        arrays[f"out_{policy}"] = torch.stack(outs).numpy()
        rec[policy] = dict(extra, anchors=flags)
    self = make_self(decode_mode="sparse", sliding_window=window)
    out, _ = ns["delta_decode_forward"](self, self, qs[0], k, v, scaling=scaling)
    arrays["out_sparse"] = out.numpy()
    rec.update(n_keys=n_keys, window=window, sink=1024, scaling=scaling, steps=steps)
    np.savez_compressed(os.path.join(out_dir, "decode_reference.npz"), meta=json.dumps(rec), **arrays)
    print("[golden] decode_reference", rec, flush=True)


# name: (s, H, Hkv, d, gamma, window, sink, seed)
TRAIN_FD_CASES = {
    "train_small": (512, 4, 1, 64, 64, 128, 32, 0),
    "train_gqa2_g32": (768, 4, 2, 64, 32, 256, 64, 1),
    "train_d128_g128": (1024, 8, 2, 128, 128, 192, 128, 2),
}
TRAIN_FD_DIRS = 3
TRAIN_FD_EPS = 1e-5


def train_fd_tensors(case, dir_index: int):
    """Inputs (float64 of the bf16-rounded synthetic q/k/v), the loss weights W
    and direction ``dir_index`` of a finite-difference case; shared with the
    test that checks the oracle's gradients against the stored values."""
    s, H, Hkv, d, gamma, window, sink, seed = case
    q, k, v = make_inputs(s, H, Hkv, d, seed=seed, rope_theta=500000.0, dtype=torch.bfloat16)
    q, k, v = q.double(), k.double(), v.double()
    g = torch.Generator().manual_seed(9000 + seed)
    w = torch.randn(1, s, H, d, generator=g, dtype=torch.float64)
    g = torch.Generator().manual_seed(9100 + 10 * seed + dir_index)
    dirs = tuple(torch.randn(t.shape, generator=g, dtype=torch.float64) for t in (q, k, v))
    return (q, k, v), w, dirs


def gen_train_fd(ref: str, out_dir: str) -> None:
    """Directional derivatives of L = sum(W * out) of the reference's own
    ``delta_forward_train`` (eager FlexAttention has no CPU backward, so central
    finite differences of its float64 forward along seeded random directions of
    (q, k, v) jointly stand in for its gradients)."""
    flex_delta = load_flex(ref)
    torch.set_num_threads(os.cpu_count() or 1)
    rec = {"eps": TRAIN_FD_EPS, "cases": {}}
    for name, case in TRAIN_FD_CASES.items():
        s, H, Hkv, d, gamma, window, sink, seed = case
        vals = []
        for i in range(TRAIN_FD_DIRS):
            (q, k, v), w, (dq, dk, dv) = train_fd_tensors(case, i)

            def loss(e):
                with torch.no_grad():
                    o = flex_delta.delta_forward_train(q + e * dq, k + e * dk, v + e * dv, gamma=gamma,
                                                       window=window, sink=sink)
                return float((o.double() * w).sum())

            vals.append((loss(TRAIN_FD_EPS) - loss(-TRAIN_FD_EPS)) / (2 * TRAIN_FD_EPS))
        rec["cases"][name] = {"case": list(case), "directional_derivatives": vals}
        print(f"[golden] train_fd {name}: {vals}", flush=True)
    with open(os.path.join(out_dir, "train_fd.json"), "w") as f:
        json.dump(rec, f, indent=1)


def gen_cpu_timing(ref: str, out_dir: str, repeats: int = 2) -> None:
    """Time the reference's own CPU path (``delta_forward_train``, eager
    FlexAttention, fp32) against this repository's CPU oracle port on the same
    config-1 input, same host and thread count.  The GPU box has no reference
    checkout, so the benchmark's reference arm times the port; this record
    relates the two (``port_over_reference`` = port tokens/s / reference tokens/s)."""
    import platform

    from oracle import delta_oracle as orc

    flex_delta = load_flex(ref)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    s, H, Hkv, d, gamma, window, sink, theta, seed, _ = FLEX_CASES["flex_config1"]
    q, k, v = make_inputs(s, H, Hkv, d, seed=seed, rope_theta=theta, dtype=torch.bfloat16)

    def best(fn):
        ts = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            with torch.no_grad():
                fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    t_ref = best(lambda: flex_delta.delta_forward_train(q.float(), k.float(), v.float(), gamma=gamma,
                                                          window=window, sink=sink))
    t_port = best(lambda: orc.delta_forward(q, k, v, gamma, window, sink, dtype=torch.float32))
    cpu = platform.processor() or platform.machine()
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), cpu)
    except OSError:
        pass
    rec = {
        "what": "whole config-1 layer (s=4096, 32/8 heads, d=128, W=1024, S=64, gamma=64), fp32 on CPU, best of "
                f"{repeats}",
        "reference": "delta_attention/train/flex_delta.py delta_forward_train (eager flex_attention)",
        "port": "oracle/delta_oracle.py delta_forward (dtype float32)",
        "host_cpu": cpu, "threads": threads, "torch": torch.__version__,
        "reference_s": t_ref, "port_s": t_port,
        "reference_tokens_per_s": s / t_ref, "port_tokens_per_s": s / t_port,
        "port_over_reference": t_ref / t_port,
    }
    with open(os.path.join(out_dir, "cpu_timing.json"), "w") as f:
        json.dump(rec, f, indent=1)
    print("[golden] cpu_timing", rec, flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DTA_REFERENCE"),
                    help="path of the reference checkout (or set DTA_REFERENCE)")
    ap.add_argument("--only", nargs="*")
    ap.add_argument("--timing-only", action="store_true",
                    help="only write cpu_timing.json (reference CPU path vs the oracle port)")
    ap.add_argument("--train-fd-only", action="store_true",
                    help="only write train_fd.json (finite differences of the reference's training forward)")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <checkout> or set DTA_REFERENCE")
    if not os.path.isdir(args.reference):
        raise SystemExit(f"reference checkout not found at {args.reference}")
    if args.timing_only:
        gen_cpu_timing(args.reference, HERE)
        return
    if args.train_fd_only:
        gen_train_fd(args.reference, HERE)
        return
    gen_stride(args.reference, HERE)
    gen_decode(args.reference, HERE)
    gen_flex(args.reference, HERE, args.only)
    gen_train_fd(args.reference, HERE)


if __name__ == "__main__":
    main()
