"""The reference-facing plug-in (DeltaAttention) on the GPU: the reference's
identity tests T2, T6, T8 and the decode refresh schedule, rectangle rows,
adaptive stride and drift telemetry."""

import types

import pytest
import torch

from delta_attention_b200.config import Config
from delta_attention_b200.synthetic import make_inputs
from oracle import delta_oracle as orc
from tests._helpers import assert_close

pytestmark = pytest.mark.gpu


def _module(**over):
    cfg = types.SimpleNamespace()
    c = Config(**{k: v for k, v in over.items() if hasattr(Config, k)})
    for f in ("mode", "delta_lambda", "sliding_window", "sink", "q_block", "log_drift", "stride_policy",
              "gamma_min", "gamma_max", "adapt_chunk", "adapt_threshold", "stride_trigger", "adapt_k",
              "decode_mode", "gamma_dec", "refresh_policy", "drift_threshold", "drift_k", "gamma_dec_max"):
        setattr(cfg, f, getattr(c, f))
    cfg.num_attention_heads = over.get("heads", 32)
    cfg.num_key_value_heads = over.get("kv_heads", 8)
    cfg.head_dim = 128
    from delta_attention_b200.attention import DeltaAttention
    return DeltaAttention(cfg, layer_idx=over.get("layer", 0))


def test_t2_anchor_exactness_via_plugin():
    m = _module(delta_lambda=64, sliding_window=2048, sink=1024)
    s = 8192
    q, k, v = make_inputs(s, 32, 8, 128, seed=0, device="cuda", gen_device="cuda")
    out, none = m.delta_forward(m, q, k, v, None, scaling=128 ** -0.5,
                                position_ids=torch.arange(s, device="cuda")[None])
    assert none is None and out.shape == (1, s, 32, 128)
    anchors, tail, _ = orc.anchor_layout(s, 64)
    rows = torch.cat((anchors[::8], tail[::16]))
    dense = orc.dense_rows(q.cpu().float(), k.cpu().float(), v.cpu().float(), rows, 128 ** -0.5)
    cos = orc.row_cos(out[:, rows.cuda()].cpu(), dense)
    assert cos.min().item() > 0.999


def _step(seed, n=8192, heads=32, kv=8):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, heads, 1, 128, generator=g).bfloat16().cuda()
    k = torch.randn(1, kv, n, 128, generator=g).bfloat16().cuda()
    v = torch.randn(1, kv, n, 128, generator=g).bfloat16().cuda()
    return q, k, v


def test_t6_anchor_step_equals_dense():
    q, k, v = _step(0)
    m = _module(decode_mode="delta", gamma_dec=8, refresh_policy="fixed", sliding_window=2048)
    out_anchor, _ = m.sdpa_rectangle_forward(m, q, k, v, scaling=128 ** -0.5)
    d = _module(decode_mode="dense")
    out_dense, _ = d.sdpa_rectangle_forward(d, q, k, v, scaling=128 ** -0.5)
    cos = torch.nn.functional.cosine_similarity(out_anchor.flatten().float(), out_dense.flatten().float(), dim=0)
    assert cos.item() > 0.999
    ref = orc.dense_decode(q.cpu().float(), k.cpu().float(), v.cpu().float(), 128 ** -0.5)
    assert_close(out_dense.cpu(), ref, "dense decode via plug-in")


def test_t8_zero_delta_is_bit_equal_sparse():
    q, k, v = _step(1)
    m = _module(decode_mode="delta", gamma_dec=10_000, refresh_policy="fixed", gamma_dec_max=100_000)
    m.sdpa_rectangle_forward(m, q, k, v, scaling=128 ** -0.5)
    m._dec_state["last_delta"] = torch.zeros_like(m._dec_state["last_delta"])
    q2, _, _ = _step(2)
    out_zero, _ = m.sdpa_rectangle_forward(m, q2, k, v, scaling=128 ** -0.5)
    sp = _module(decode_mode="sparse")
    out_sparse, _ = sp.sdpa_rectangle_forward(sp, q2, k, v, scaling=128 ** -0.5)
    assert torch.equal(out_zero, out_sparse)


def test_decode_refresh_schedule_and_per_layer_state():
    m0 = _module(decode_mode="delta", gamma_dec=2, refresh_policy="fixed", gamma_dec_max=100, log_drift=True)
    m1 = _module(decode_mode="delta", gamma_dec=2, refresh_policy="fixed", gamma_dec_max=100, log_drift=True,
                 layer=1)
    flags, steps = [], []
    for seed in (10, 11, 12):
        q, k, v = _step(seed)
        m0.sdpa_rectangle_forward(m0, q, k, v, scaling=128 ** -0.5)
        flags.append(m0._dec_drift_points[-1]["anchor"])
        steps.append(m0._dec_state["steps"])
    assert flags == [True, False, True]
    assert steps == [0, 1, 0]
    assert m1._dec_state is None
    q, k, v = _step(13)
    m1.sdpa_rectangle_forward(m1, q, k, v, scaling=128 ** -0.5)
    assert m1._dec_drift_points[-1]["anchor"] is True
    assert m1._dec_state is not m0._dec_state


def test_delta_decode_matches_oracle_sequence():
    """Several delta-decode steps (fixed policy) vs the oracle's state machine."""
    g = torch.Generator().manual_seed(5)
    k = torch.randn(1, 8, 5000, 128, generator=g).bfloat16()
    v = torch.randn(1, 8, 5000, 128, generator=g).bfloat16()
    m = _module(decode_mode="delta", gamma_dec=3, refresh_policy="fixed", sliding_window=1024, sink=1024)
    st = orc.OracleDecodeState()
    for t in range(7):
        q = torch.randn(1, 32, 1, 128, generator=g).bfloat16()
        out, _ = m.sdpa_rectangle_forward(m, q.cuda(), k.cuda(), v.cuda(), scaling=128 ** -0.5)
        ref, anchor = orc.delta_decode_step(st, q.float(), k.float(), v.float(), window=1024, sink=1024,
                                            scaling=128 ** -0.5, gamma_dec=3)
        assert (m._dec_state["steps"] == 0) == anchor
        assert_close(out.cpu(), ref, f"delta decode step {t}", max_abs=2e-2)


def test_rectangle_rows_s_gt_1():
    s_new, n = 5, 3000
    q, k, v = make_inputs(n, 32, 8, 128, seed=3)
    qn = q[:, :, -s_new:]
    m = _module(decode_mode="dense")
    out, _ = m.sdpa_rectangle_forward(m, qn.cuda(), k.cuda(), v.cuda(), scaling=128 ** -0.5)
    lim = torch.arange(n - s_new, n)
    ref = orc.dense_rows(qn.float().contiguous(), k.float(), v.float(), torch.arange(s_new), 128 ** -0.5, limits=lim)
    assert_close(out.cpu(), ref, "rectangle rows")


def test_adaptive_stride_matches_variable_oracle():
    s = 4096
    q, k, v = make_inputs(s, 8, 2, 128, seed=7)
    m = _module(delta_lambda=64, sliding_window=512, sink=64, stride_policy="adaptive", adapt_chunk=1024,
                adapt_threshold=0.5, gamma_min=16, gamma_max=256, heads=8, kv_heads=2)
    out, _ = m.delta_forward(m, q.cuda(), k.cuda(), v.cuda(), None, scaling=128 ** -0.5)
    stats = m._stride_stats
    assert stats is not None and stats["chunks"]
    idx = torch.cat([torch.arange(c["start"], min(c["start"] + 1024, s - 128), c["gamma"]) for c in stats["chunks"]])
    assert idx.numel() == stats["n_anchors"]
    ref = orc.delta_forward_variable(q.float(), k.float(), v.float(), idx, 512, 64, s - 128)
    assert_close(out.cpu(), ref, "adaptive stride")


def test_log_drift_summary():
    m = _module(delta_lambda=64, sliding_window=256, sink=32, log_drift=True, heads=8, kv_heads=2)
    q, k, v = make_inputs(2048, 8, 2, 128, seed=8)
    m.delta_forward(m, q.cuda(), k.cuda(), v.cuda(), None, scaling=128 ** -0.5)
    st = m._drift_stats
    assert st["n"] == ((2048 - 128) // 64 - 1) * 8  # consecutive-anchor pairs x heads
    assert sum(st["hist"]) > 0 and -1.0 <= st["mean"] <= 1.0


@pytest.mark.parametrize("policy,extra", [("drift", dict(drift_threshold=0.95)),
                                          ("drift_rel", dict(drift_k=50.0))])
def test_drift_refresh_policies_match_oracle(policy, extra):
    """delta-mode decode with a drift-triggered refresh (``delta_attention/llama.py:586-606``):
    the anchor decision needs this step's sparse row first, so the plug-in runs
    the sparse pass, decides, and reads the dense row only on an anchor.  A
    query sequence that drifts slowly and then jumps once must give the
    oracle's anchor flags and outputs step by step."""
    n0, T, H, Hkv, d = 4096, 14, 32, 8, 128
    g = torch.Generator().manual_seed(11)
    k = torch.randn(1, Hkv, n0 + T, d, generator=g).bfloat16()
    v = torch.randn(1, Hkv, n0 + T, d, generator=g).bfloat16()
    q0 = torch.randn(1, H, 1, d, generator=g)
    dq = torch.randn(1, H, 1, d, generator=g)
    jump = torch.randn(1, H, 1, d, generator=g)
    qs = [((jump if t >= 11 else q0) + 0.02 * t * dq).bfloat16() for t in range(T)]
    m = _module(decode_mode="delta", refresh_policy=policy, gamma_dec=64, gamma_dec_max=128,
                sliding_window=1024, sink=128, **extra)
    st = orc.OracleDecodeState()
    flags, ref_flags = [], []
    for t in range(T):
        n = n0 + t
        kc, vc = k[:, :, :n + 1], v[:, :, :n + 1]
        out, _ = m.sdpa_rectangle_forward(m, qs[t].cuda(), kc.cuda(), vc.cuda(), scaling=d ** -0.5)
        flags.append(m._dec_state["steps"] == 0)
        ref, a = orc.delta_decode_step(st, qs[t].float(), kc.float(), vc.float(), window=1024, sink=128,
                                       scaling=d ** -0.5, gamma_dec=64, refresh_policy=policy,
                                       drift_k=extra.get("drift_k", 2.0),
                                       drift_threshold=extra.get("drift_threshold", 0.95), gamma_dec_max=128)
        ref_flags.append(a)
        assert_close(out.cpu(), ref, f"{policy} step {t}")
    assert flags == ref_flags, (flags, ref_flags)
    assert flags[0] and flags[11] and sum(flags) == 2, flags  # first step and the jump
