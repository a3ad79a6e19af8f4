"""Tensor-parallel Llama-3.1 / Qwen3 decoder whose attention is the delta plug-in.

The end-to-end workload around the attention path (BASELINE configs 3 and 4):
random-init bf16 weights of the Llama-3.1-8B or Qwen3-8B architecture, a
prefill of the prompt with delta attention in every layer, then greedy decode
with dense, sparse or delta-mode attention.  The layer follows the reference's
patched model:

* attention forward: q/k/v projections (``_qkv`` hook), RoPE, KV-cache
  update, plug-in attention, o_proj (``delta_attention/llama.py:826-914``;
  cache update ``:857-862``);
* Qwen3: per-head RMSNorm of q and k before RoPE (``delta_attention/qwen3.py:30-43``);
* MLP: ``down(silu(gate(x)) * up(x))`` (``delta_attention/llama.py:195-215``);
* prefill -> decode switch: a new prompt resets every layer's decode state,
  prefill runs the delta path, later steps the decode path
  (``delta_attention/sample.py:145-161``).

Parallelism (one process per GPU): every rank owns ``n_kv_heads / world`` whole
KV groups and the query heads of those groups, so attention runs locally with
no collective (the same partition as the single-layer benchmark).  QKV and the
MLP gate/up projections are column-parallel, o_proj and down row-parallel, each
followed by an all-reduce of the hidden states (NCCL over NVLink); the LM head
is split over the vocabulary and the next token is a global argmax.  The
embedding is replicated.  GEMMs are plain library GEMMs (torch / cuBLAS).
"""

from __future__ import annotations

import dataclasses
import zlib
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch

from .attention import DeltaAttention
from .config import PIPELINE_FIELDS, Config
from .rope import cos_sin, rotate_half


@dataclass(frozen=True)
class Arch:
    name: str
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float
    rope_theta: float
    rope_llama3: Optional[Tuple[Tuple[str, float], ...]]  # llama3 frequency schedule, as items
    qk_norm: bool


LLAMA31_8B = Arch("llama-3.1-8b", 32, 4096, 32, 8, 128, 14336, 128256, 1e-5, 500000.0,
                  (("factor", 8.0), ("low_freq_factor", 1.0), ("high_freq_factor", 4.0),
                   ("original_max_position_embeddings", 8192.0)), False)
QWEN3_8B = Arch("qwen3-8b", 36, 4096, 32, 8, 128, 12288, 151936, 1e-6, 1000000.0, None, True)
ARCHS = {"llama": LLAMA31_8B, "qwen3": QWEN3_8B}


def tiny(arch: Arch, **kw) -> Arch:
    """A small model of the same family (tests)."""
    return dataclasses.replace(arch, **kw)


class TP:
    """Rank, world and process group of the tensor-parallel job (world 1: none)."""

    def __init__(self, rank: int = 0, world: int = 1, group=None):
        self.rank, self.world, self.group = rank, world, group

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            torch.distributed.all_reduce(t, group=self.group)
        return t

    def all_gather(self, t: torch.Tensor) -> List[torch.Tensor]:
        if self.world == 1:
            return [t]
        out = [torch.empty_like(t) for _ in range(self.world)]
        torch.distributed.all_gather(out, t, group=self.group)
        return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm in fp32, result in x's dtype (LlamaRMSNorm)."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * xf).to(x.dtype)


class _PluginConfig:
    """Per-rank view of the model config the plug-in reads: local head counts
    plus the pipeline knobs of a :class:`Config`."""

    def __init__(self, cfg: Config, n_heads: int, n_kv_heads: int, head_dim: int):
        for f in PIPELINE_FIELDS:
            setattr(self, f, getattr(cfg, f))
        self.num_attention_heads = n_heads
        self.num_key_value_heads = n_kv_heads
        self.head_dim = head_dim


# An attention override (tests on CPU): (layer, q [B,H,s,d], k, v [B,Hkv,n,d],
# scaling, prefill) -> [B, s, H, d].
AttentionFn = Callable[[int, torch.Tensor, torch.Tensor, torch.Tensor, float, bool], torch.Tensor]


class DeltaDecoder:
    """The tensor-parallel decoder of one rank (weights, KV cache, plug-ins)."""

    def __init__(self, arch: Arch, cfg: Config, tp: Optional[TP] = None, device="cuda",
                 dtype: torch.dtype = torch.bfloat16, seed: int = 0, attention: Optional[AttentionFn] = None,
                 init_std: float = 0.02):
        self.arch, self.cfg, self.tp = arch, cfg, tp or TP()
        self.device, self.dtype = torch.device(device), dtype
        W, r = self.tp.world, self.tp.rank
        if arch.n_kv_heads % W or arch.intermediate % W or arch.vocab % W:
            raise ValueError(f"world {W} must divide the KV heads, the MLP width and the vocabulary")
        self.Hl, self.Hkvl = arch.n_heads // W, arch.n_kv_heads // W
        self.Il, self.Vl = arch.intermediate // W, arch.vocab // W
        d, D = arch.head_dim, arch.hidden
        self.scaling = d ** -0.5
        self.attention = attention
        self.events: Optional[Dict[str, List]] = None  # phase timing (set by the benchmark)

        # Weights: every rank draws the FULL tensor from a generator seeded by
        # (seed, layer, name) and keeps its slice, so the model is the same
        # function of its seed at any world size.
        gdev = self.device if self.device.type == "cuda" else torch.device("cpu")

        def draw(shape, key, std=init_std):
            g = torch.Generator(device=gdev).manual_seed(zlib.crc32(repr((seed,) + key).encode()))
            return (torch.randn(*shape, generator=g, device=gdev, dtype=torch.float32) * std)

        def rows(w, lo, n):
            return w[lo:lo + n]

        self.embed = draw((arch.vocab, D), ("embed",)).to(dtype)
        self.final_norm = torch.ones(D, device=self.device, dtype=dtype)
        self.lm_head = rows(draw((arch.vocab, D), ("lm_head",)), r * self.Vl, self.Vl).to(dtype).contiguous()
        self.layers = []
        for i in range(arch.n_layers):
            wq = draw((arch.n_heads * d, D), (i, "q"))
            wk = draw((arch.n_kv_heads * d, D), (i, "k"))
            wv = draw((arch.n_kv_heads * d, D), (i, "v"))
            # column-parallel: this rank's query heads and KV heads, one fused GEMM
            w_qkv = torch.cat((rows(wq, r * self.Hl * d, self.Hl * d), rows(wk, r * self.Hkvl * d, self.Hkvl * d),
                               rows(wv, r * self.Hkvl * d, self.Hkvl * d))).to(dtype).contiguous()
            del wq, wk, wv
            # row-parallel o_proj: the input columns of this rank's heads
            w_o = draw((D, arch.n_heads * d), (i, "o"))[:, r * self.Hl * d:(r + 1) * self.Hl * d].to(dtype).contiguous()
            wg = draw((arch.intermediate, D), (i, "gate"))
            wu = draw((arch.intermediate, D), (i, "up"))
            w_gu = torch.cat((rows(wg, r * self.Il, self.Il), rows(wu, r * self.Il, self.Il))).to(dtype).contiguous()
            del wg, wu
            w_down = draw((D, arch.intermediate), (i, "down"))[:, r * self.Il:(r + 1) * self.Il].to(dtype).contiguous()
            layer = {"w_qkv": w_qkv, "w_o": w_o, "w_gu": w_gu, "w_down": w_down,
                     "norm1": torch.ones(D, device=self.device, dtype=dtype),
                     "norm2": torch.ones(D, device=self.device, dtype=dtype)}
            if arch.qk_norm:
                layer["q_norm"] = torch.ones(d, device=self.device, dtype=dtype)
                layer["k_norm"] = torch.ones(d, device=self.device, dtype=dtype)
            layer["plugin"] = DeltaAttention(_PluginConfig(cfg, self.Hl, self.Hkvl, d), layer_idx=i)
            self.layers.append(layer)
        self.k_cache: List[torch.Tensor] = []
        self.v_cache: List[torch.Tensor] = []
        self.length = 0
        llama3 = dict(arch.rope_llama3) if arch.rope_llama3 else None
        self._rope = (arch.head_dim, arch.rope_theta, llama3)

    # ------------------------------------------------------------------
    def allocate_cache(self, batch: int, max_len: int) -> None:
        """KV cache [B, KV heads of this rank, max_len, d] per layer, bf16."""
        shape = (batch, self.Hkvl, max_len, self.arch.head_dim)
        self.k_cache = [torch.empty(shape, device=self.device, dtype=self.dtype) for _ in self.layers]
        self.v_cache = [torch.empty(shape, device=self.device, dtype=self.dtype) for _ in self.layers]
        self.length = 0

    def _timed(self, name: str):
        """CUDA-event bracket around one phase of a layer (benchmark only)."""
        ev = self.events
        if ev is None:
            return _NullCtx()
        return _EventCtx(ev.setdefault(name, []))

    def _attend(self, i: int, layer, q, k, v, prefill: bool) -> torch.Tensor:
        if self.attention is not None:
            return self.attention(i, q, k, v, self.scaling, prefill)
        plug = layer["plugin"]
        if prefill:
            out, _ = plug.delta_forward(plug, q, k, v, None, scaling=self.scaling)
        else:
            out, _ = plug.sdpa_rectangle_forward(plug, q, k, v, None, scaling=self.scaling)
        return out

    def _layer(self, i: int, x: torch.Tensor, pos0: int, cos: torch.Tensor, sin: torch.Tensor,
               pos_t: Optional[torch.Tensor] = None, attend: Optional[Callable] = None) -> torch.Tensor:
        """One decoder layer.  ``pos_t`` (a device position, one new token)
        and ``attend(i, q, k_cache, v_cache)`` select the graph-replayed decode
        step: the cache write and the attention then take the position from
        device memory and the attention reads the whole cache."""
        a, layer = self.arch, self.layers[i]
        B, s, D = x.shape
        d = a.head_dim
        with self._timed("gemm"):
            h = rms_norm(x, layer["norm1"], a.rms_eps)
            qkv = h @ layer["w_qkv"].t()
        q, k, v = qkv.split((self.Hl * d, self.Hkvl * d, self.Hkvl * d), dim=-1)
        q = q.view(B, s, self.Hl, d)
        k = k.view(B, s, self.Hkvl, d)
        v = v.view(B, s, self.Hkvl, d)
        if a.qk_norm:  # Qwen3's _qkv hook
            q = rms_norm(q, layer["q_norm"], a.rms_eps)
            k = rms_norm(k, layer["k_norm"], a.rms_eps)
        # RoPE in the activations' dtype with cos/sin rounded to it, as the
        # reference's layers do (``delta_attention/llama.py:183-192``)
        c, sn = cos[:, None, :].to(q.dtype), sin[:, None, :].to(q.dtype)
        q = q * c + rotate_half(q) * sn
        k = k * c + rotate_half(k) * sn
        # KV-cache write path: post-RoPE keys and values at positions [pos0, pos0 + s)
        kc, vc = self.k_cache[i], self.v_cache[i]
        if pos_t is not None:
            kc.index_copy_(2, pos_t, k.transpose(1, 2))
            vc.index_copy_(2, pos_t, v.transpose(1, 2))
            o = attend(i, q.transpose(1, 2), kc, vc)
        else:
            kc[:, :, pos0:pos0 + s] = k.transpose(1, 2)
            vc[:, :, pos0:pos0 + s] = v.transpose(1, 2)
            n = pos0 + s
            with self._timed("attention"):
                o = self._attend(i, layer, q.transpose(1, 2), kc[:, :, :n], vc[:, :, :n], prefill=(pos0 == 0))
        with self._timed("gemm"):
            o = o.reshape(B, s, self.Hl * d) @ layer["w_o"].t()
        with self._timed("all_reduce"):
            x = x + self.tp.all_reduce(o)
        with self._timed("gemm"):
            h = rms_norm(x, layer["norm2"], a.rms_eps)
            gu = h @ layer["w_gu"].t()
            g, u = gu.split(self.Il, dim=-1)
            m = (torch.nn.functional.silu(g) * u) @ layer["w_down"].t()
        with self._timed("all_reduce"):
            x = x + self.tp.all_reduce(m)
        return x

    def _next_token(self, x_last: torch.Tensor) -> torch.Tensor:
        """Greedy next token from the last position's hidden state [B, D]."""
        h = rms_norm(x_last, self.final_norm, self.arch.rms_eps)
        logits = (h @ self.lm_head.t()).float()  # [B, vocab / world]
        val, idx = logits.max(dim=-1)
        idx = idx + self.tp.rank * self.Vl
        if self.tp.world == 1:
            return idx
        vals = torch.stack(self.tp.all_gather(val.contiguous()))   # [W, B]
        idxs = torch.stack(self.tp.all_gather(idx.contiguous()))
        best = vals.argmax(dim=0)
        return idxs.gather(0, best[None]).squeeze(0)

    def logits_last(self, x_last: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits of the last position (tests)."""
        h = rms_norm(x_last, self.final_norm, self.arch.rms_eps)
        return torch.cat(self.tp.all_gather((h @ self.lm_head.t()).float().contiguous()), dim=-1)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Run the next ``s`` positions (prefill when the cache is empty);
        returns the hidden states [B, s, D] after the last layer."""
        B, s = input_ids.shape
        pos0 = self.length
        if pos0 == 0:
            for layer in self.layers:  # a new prompt: no decode state carries over
                layer["plugin"].reset_decode_state()
        if pos0 + s > (self.k_cache[0].shape[2] if self.k_cache else 0):
            raise ValueError("KV cache too short: call allocate_cache(batch, max_len) first")
        x = self.embed[input_ids.to(self.embed.device)]
        cos, sin = cos_sin(torch.arange(pos0, pos0 + s, device=self.device), *self._rope)
        for i in range(len(self.layers)):
            x = self._layer(i, x, pos0, cos, sin)
        self.length = pos0 + s
        return x

    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Prompt [B, N] -> first generated token [B]."""
        self.length = 0
        return self._next_token(self.forward(input_ids)[:, -1])

    def decode_step(self, tokens: torch.Tensor) -> torch.Tensor:
        """One new token per sequence [B] -> the next token [B]."""
        return self._next_token(self.forward(tokens[:, None])[:, -1])


class DecodeGraph:
    """Greedy decode with one CUDA-graph replay per token.

    One decode step of the whole model (every layer's projections, RoPE,
    KV-cache write, attention, all-reduces, the LM head and the next-token
    choice) is captured once and replayed; the input token, the position and
    the live cache length are device tensors that the graph advances itself,
    so the host issues one replay per token instead of hundreds of launches.
    The attention is the plug-in's decode kernel with the key count read from
    device memory (``ops.decode(..., n_keys_dev=)``) over the whole cache.
    Modes: dense, sparse, and delta with the fixed refresh schedule (anchor
    every ``min(gamma_dec, gamma_dec_max)`` steps, ``delta_attention/llama.py:552-634``):
    delta mode captures an anchor step (dense and sparse rows, delta refreshed,
    output = dense) and a sparse step (output = sparse + delta), and the host
    picks the graph by the step count.  Drift policies and drift logging
    decide from device values on the host and use the eager path
    (:meth:`DeltaDecoder.decode_step`)."""

    def __init__(self, model: "DeltaDecoder", batch: int):
        cfg = model.cfg
        self.model, self.batch = model, batch
        self.mode = getattr(cfg, "decode_mode", "dense")
        if self.mode == "delta" and (getattr(cfg, "refresh_policy", "fixed") != "fixed"
                                     or getattr(cfg, "log_drift", False)):
            raise ValueError("graph decode supports the fixed refresh schedule without drift logging")
        self.period = max(1, min(int(getattr(cfg, "gamma_dec", 32)), int(getattr(cfg, "gamma_dec_max", 128))))
        self.window = int(cfg.sliding_window)
        self.sink = int(getattr(cfg, "sink", 1024))
        dev, d = model.device, model.arch.head_dim
        self.tok = torch.zeros(batch, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.n_keys = torch.zeros(1, dtype=torch.int32, device=dev)
        self.hidden = torch.zeros(batch, model.arch.hidden, dtype=model.dtype, device=dev)  # last step's output
        self.delta = [torch.zeros(batch, 1, model.Hl, d, dtype=torch.bfloat16, device=dev) for _ in model.layers] \
            if self.mode == "delta" else []
        self.graphs: Dict[bool, torch.cuda.CUDAGraph] = {}
        self.steps = 0

    def _attend(self, anchor: bool):
        from . import ops

        m = self.model

        def attend(i, q, kc, vc):
            kw = dict(window=self.window, sink=self.sink, scaling=m.scaling, n_keys_dev=self.n_keys)
            if self.mode == "dense":
                out, _ = ops.decode(q, kc, vc, want_dense=True, want_sparse=False, **kw)
            elif self.mode == "sparse":
                _, out = ops.decode(q, kc, vc, want_dense=False, want_sparse=True, **kw)
            elif anchor:
                dense, sparse = ops.decode(q, kc, vc, want_dense=True, want_sparse=True, **kw)
                self.delta[i].copy_(dense - sparse)
                out = dense
            else:
                _, sparse = ops.decode(q, kc, vc, want_dense=False, want_sparse=True, **kw)
                out = sparse + self.delta[i]
            return out

        return attend

    def _step(self, anchor: bool) -> None:
        m = self.model
        x = m.embed[self.tok][:, None, :]
        cos, sin = cos_sin(self.pos, *m._rope)
        attend = self._attend(anchor)
        for i in range(len(m.layers)):
            x = m._layer(i, x, 0, cos, sin, pos_t=self.pos, attend=attend)
        self.hidden.copy_(x[:, -1])
        self.tok.copy_(m._next_token(x[:, -1]))
        self.pos.add_(1)
        self.n_keys.add_(1)

    def _capture(self) -> None:
        saved = (self.tok.clone(), self.pos.clone(), self.n_keys.clone())
        for anchor in ((True, False) if self.mode == "delta" else (False,)):
            # one eager run first (kernel attributes, library handles, NCCL
            # communicators), then rewind the device state it advanced; the
            # cache slot it wrote is written again by the first real step
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._step(anchor)
            torch.cuda.current_stream().wait_stream(side)
            for t, v in zip((self.tok, self.pos, self.n_keys), saved):
                t.copy_(v)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._step(anchor)
            self.graphs[anchor] = g

    def start(self, first_token: torch.Tensor) -> None:
        """Begin decoding after :meth:`DeltaDecoder.prefill` (which returned
        ``first_token``): the next step writes cache position ``model.length``."""
        m = self.model
        self.tok.copy_(first_token)
        self.pos.fill_(m.length)
        self.n_keys.fill_(m.length + 1)
        self.steps = 0
        if not self.graphs:
            self._capture()

    def step(self) -> torch.Tensor:
        """One token per sequence; returns the device tensor of the next token
        (overwritten by the next step)."""
        anchor = self.mode == "delta" and self.steps % self.period == 0
        self.graphs[anchor].replay()
        self.steps += 1
        self.model.length += 1
        return self.tok

    def release(self) -> None:
        """Drop the graphs (before a process group that they use is destroyed)."""
        self.graphs.clear()


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class _EventCtx:
    def __init__(self, sink: List):
        self.sink = sink

    def __enter__(self):
        self.e0 = torch.cuda.Event(enable_timing=True)
        self.e0.record()
        return self

    def __exit__(self, *a):
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        self.sink.append((self.e0, e1))
        return False
