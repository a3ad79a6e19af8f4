"""GPU parity of the sm_100a prefill kernels against the CPU oracle (which is
itself pinned to the reference's outputs by test_oracle_golden.py)."""

import json
import os

import numpy as np
import pytest
import torch

from delta_attention_b200.synthetic import make_inputs
from oracle import delta_oracle as orc
from tests._helpers import MAX_ABS, assert_close

pytestmark = pytest.mark.gpu


def _run(q, k, v, **kw):
    from delta_attention_b200 import ops
    return ops.prefill(q.cuda(), k.cuda(), v.cuda(), **kw)


def _oracle_full(q, k, v, gamma, window, sink, mode="delta"):
    return orc.delta_forward(q.float(), k.float(), v.float(), gamma, window, sink, mode=mode)


@pytest.mark.parametrize("s,H,Hkv,d,gamma,window,sink", [
    (1024, 4, 1, 128, 64, 256, 64),     # GQA 4 (R = 32 rows x 4 heads)
    (1024, 8, 2, 128, 16, 192, 32),     # gamma 16
    (768, 2, 2, 128, 32, 128, 16),      # no GQA (R = 128)
    (1024, 8, 1, 128, 128, 256, 128),   # GQA 8, gamma 128
    (640, 4, 2, 64, 64, 128, 64),       # head_dim 64
    (1000, 4, 1, 128, 8, 300, 50),      # ragged length, odd window/sink
])
def test_prefill_delta_matches_oracle(s, H, Hkv, d, gamma, window, sink):
    q, k, v = make_inputs(s, H, Hkv, d, seed=s + gamma)
    out = _run(q, k, v, gamma=gamma, window=window, sink=sink)
    torch.cuda.synchronize()
    ref = _oracle_full(q, k, v, gamma, window, sink)
    assert_close(out.cpu(), ref, f"delta s={s} H={H}/{Hkv} d={d} g={gamma} W={window} S={sink}")


@pytest.mark.parametrize("batch,Hkv", [(2, 2), (3, 1)])
def test_prefill_batched_sequences(batch, Hkv):
    """Several sequences in one call: every (sequence, KV group) pair is its own
    set of jobs (the layout the benchmark uses to stack a rank's units)."""
    s, d, gamma, window, sink = 768, 128, 64, 192, 64
    H = 4 * Hkv
    q, k, v = make_inputs(s, H, Hkv, d, seed=7 + batch, batch=batch)
    out = _run(q, k, v, gamma=gamma, window=window, sink=sink)
    torch.cuda.synchronize()
    ref = _oracle_full(q, k, v, gamma, window, sink)
    assert_close(out.cpu(), ref, f"batch {batch} Hkv {Hkv}")


@pytest.mark.parametrize("mode,s", [("sparse-only", 1024), ("recompute", 1024),
                                    ("sparse-only", 1000), ("recompute", 1000)])
def test_prefill_modes(mode, s):
    """s=1000: the last job's second query tile is partial, so one job mixes a
    tile stored by TMA (sparse-only) with a tile stored row by row."""
    H, Hkv, d, gamma, window, sink = 4, 1, 128, 8, 256, 64
    q, k, v = make_inputs(s, H, Hkv, d, seed=3)
    out = _run(q, k, v, gamma=gamma, window=window, sink=sink, mode=mode)
    ref = _oracle_full(q, k, v, gamma, window, sink, mode=mode)
    assert_close(out.cpu(), ref, f"mode {mode}")


GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["flex_small_gqa4", "flex_g16_d128", "flex_gamma1", "flex_fullwindow",
                                  "flex_gqa8_g128", "flex_g32_w64", "flex_config1"])
def test_prefill_matches_reference_golden(name):
    """Kernel output vs the reference's own output (flex_delta.delta_forward_train, fp32)."""
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    m = json.loads(str(z["meta"]))
    theta = None if m["rope_theta"] < 0 else m["rope_theta"]
    q, k, v = make_inputs(m["s"], m["H"], m["Hkv"], m["d"], seed=m["seed"], rope_theta=theta)
    out = _run(q, k, v, gamma=m["gamma"], window=m["window"], sink=m["sink"])
    rows = torch.from_numpy(z["rows"]).long()
    ref = torch.from_numpy(z["out"]).unsqueeze(0)
    assert_close(out.cpu()[:, rows], ref, f"golden {name}")


def test_identities_gamma1_is_dense_and_full_window():
    s, H, Hkv, d = 1024, 4, 1, 128
    q, k, v = make_inputs(s, H, Hkv, d, seed=9)
    # gamma = 1: every row below s_p is an anchor -> dense everywhere (reference T3)
    out = _run(q, k, v, gamma=1, window=128, sink=16)
    dense = orc.dense_rows(q.float(), k.float(), v.float(), torch.arange(s), d ** -0.5)
    assert_close(out.cpu(), dense, "gamma=1 vs dense")
    # window >= s: sparse == dense, delta ~ 0 (reference T4)
    out_w, delta = _run(q, k, v, gamma=64, window=s, sink=16, return_anchor_delta=True)
    assert_close(out_w.cpu(), dense, "full window vs dense")
    rel = delta.norm().item() / out_w.float().norm().item()
    assert rel < 1e-2, rel


@pytest.mark.parametrize("batch,Hkv,d", [(1, 2, 128), (2, 1, 128), (1, 2, 64)])
def test_fused_anchor_delta_matches_oracle(batch, Hkv, d):
    """gamma = 64 with 4 query heads per KV head: the windowed launch forms the
    anchors' sparse rows and dense - sparse itself; the fp32 telemetry it writes
    must match the oracle's dense minus sparse rows at every anchor."""
    s, gamma, window, sink = 1024, 64, 256, 64
    H = 4 * Hkv
    q, k, v = make_inputs(s, H, Hkv, d, seed=31 + batch, batch=batch)
    out, delta = _run(q, k, v, gamma=gamma, window=window, sink=sink, return_anchor_delta=True)
    torch.cuda.synchronize()
    anchors, _, _ = orc.anchor_layout(s, gamma)
    sc = d ** -0.5
    qf, kf, vf = q.float(), k.float(), v.float()
    ref = orc.dense_rows(qf, kf, vf, anchors, sc) - orc.sparse_rows(qf, kf, vf, anchors, window, sink, sc)
    assert_close(delta.cpu(), ref, "fused anchor delta")
    assert_close(out.cpu(), _oracle_full(q, k, v, gamma, window, sink), "fused delta output")


def test_anchor_rows_equal_dense():
    """Reference T2: anchor and tail rows of the corrected output equal dense."""
    s, H, Hkv, d, gamma = 2048, 8, 2, 128, 64
    q, k, v = make_inputs(s, H, Hkv, d, seed=4)
    out = _run(q, k, v, gamma=gamma, window=512, sink=64).cpu()
    anchors, tail, _ = orc.anchor_layout(s, gamma)
    sel = torch.cat((anchors, tail))
    dense = orc.dense_rows(q.float(), k.float(), v.float(), sel, d ** -0.5)
    assert_close(out[:, sel], dense, "anchor+tail rows vs dense")


def test_noncontiguous_token_major_inputs():
    """q/k/v as the reference's attention receives them: [b, s, h, d] storage viewed as [b, h, s, d]."""
    s, H, Hkv, d, gamma, window, sink = 1024, 8, 2, 128, 32, 256, 64
    q, k, v = make_inputs(s, H, Hkv, d, seed=12)
    qt = q.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    kt = k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    vt = v.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    from delta_attention_b200 import ops
    out = ops.prefill(qt, kt, vt, gamma=gamma, window=window, sink=sink)
    ref = _oracle_full(q, k, v, gamma, window, sink)
    assert_close(out.cpu(), ref, "token-major strides")


def test_variable_anchors():
    s, H, Hkv, d, window, sink = 1024, 4, 1, 128, 192, 32
    q, k, v = make_inputs(s, H, Hkv, d, seed=21)
    s_p = 896
    anchors = torch.tensor([0, 16, 48, 64, 200, 256, 257, 400, 512, 600, 768, 800, 895])
    from delta_attention_b200 import ops
    out = ops.prefill(q.cuda(), k.cuda(), v.cuda(), gamma=64, window=window, sink=sink, anchors=anchors, s_p=s_p)
    ref = orc.delta_forward_variable(q.float(), k.float(), v.float(), anchors, window, sink, s_p)
    assert_close(out.cpu(), ref, "variable anchors")


def test_rows_op_matches_dense_rows():
    s, H, Hkv, d = 1536, 8, 2, 128
    q, k, v = make_inputs(s, H, Hkv, d, seed=5)
    rows = torch.tensor([0, 1, 7, 100, 129, 500, 777, 1000, 1001, 1535])
    from delta_attention_b200 import ops
    out = ops.rows(q.cuda(), k.cuda(), v.cuda(), rows, rows)
    ref = orc.dense_rows(q.float(), k.float(), v.float(), rows, d ** -0.5)
    assert_close(out.cpu(), ref, "rows op")


def test_large_config2_rows_sample():
    """Config-2 shape at N=32768 (32/8 heads, W=2048, S=128, gamma=64): sampled rows vs oracle."""
    s, H, Hkv, d, gamma, window, sink = 32768, 32, 8, 128, 64, 2048, 128
    q, k, v = make_inputs(s, H, Hkv, d, seed=0, gen_device="cuda", device="cuda")
    from delta_attention_b200 import ops
    out = ops.prefill(q, k, v, gamma=gamma, window=window, sink=sink)
    g = torch.Generator().manual_seed(0)
    rows = torch.unique(torch.cat((torch.randint(0, s, (24,), generator=g),
                                   torch.tensor([0, 63, 64, 65, 2047, 2048, 32639, 32640, 32767]))))
    ref = orc.delta_forward_rows(q.cpu().float(), k.cpu().float(), v.cpu().float(), rows, gamma, window, sink)
    assert_close(out[:, rows.cuda()].cpu(), ref, "config2 N=32768 rows")


def test_error_status_raises():
    from delta_attention_b200 import ops
    from delta_attention_b200._lib import DtaError
    q, k, v = make_inputs(1000, 4, 1, 128, seed=1, device="cuda")
    with pytest.raises(DtaError, match="GAMMA"):
        ops.prefill(q, k, v, gamma=48, window=128, sink=16)


@pytest.mark.parametrize("s,H,Hkv,d,gamma,window,sink,split", [
    (2048, 8, 2, 128, 64, 256, 64, 1),     # fused delta, every dense row tile split per key tile
    (2048, 8, 1, 128, 16, 384, 32, 3),     # GQA 8, gamma 16 (sparse anchor jobs + delta kernel)
    (1536, 16, 2, 128, 128, 256, 128, 2),  # GQA 8, gamma 128
    (2000, 4, 1, 128, 8, 300, 50, 5),      # ragged length: partial last row tile
    (1280, 8, 2, 64, 32, 256, 64, 2),      # head_dim 64
])
def test_split_dense_rows_match_oracle(s, H, Hkv, d, gamma, window, sink, split):
    """Split-K of the dense rows forced at small sizes: each row tile's keys run
    as several chunks whose partials the last chunk merges.  The result must
    match the oracle and the unsplit kernel (split_tiles larger than any row)."""
    q, k, v = make_inputs(s, H, Hkv, d, seed=40 + split + gamma)
    out, delta = _run(q, k, v, gamma=gamma, window=window, sink=sink, split_tiles=split,
                      return_anchor_delta=True)
    whole, delta_whole = _run(q, k, v, gamma=gamma, window=window, sink=sink, split_tiles=1 << 20,
                              return_anchor_delta=True)
    torch.cuda.synchronize()
    from delta_attention_b200 import ops
    ops.check_errors()
    ref = _oracle_full(q, k, v, gamma, window, sink)
    assert_close(out.cpu(), ref, f"split {split}: s={s} H={H}/{Hkv} d={d} g={gamma}")
    assert_close(out.cpu(), whole.cpu(), f"split {split} vs unsplit")
    assert_close(delta.cpu(), delta_whole.cpu(), f"split {split} anchor delta vs unsplit")


def test_rows_op_split_matches_dense_rows():
    """dta_rows with one key tile per chunk: long rows merge up to 12 partials."""
    s, H, Hkv, d = 1536, 8, 2, 128
    q, k, v = make_inputs(s, H, Hkv, d, seed=15)
    rows = torch.tensor([0, 5, 127, 128, 300, 777, 1000, 1200, 1400, 1535])
    from delta_attention_b200 import ops
    out = ops.rows(q.cuda(), k.cuda(), v.cuda(), rows, rows, split_tiles=1, check=True)
    ref = orc.dense_rows(q.float(), k.float(), v.float(), rows, d ** -0.5)
    assert_close(out.cpu(), ref, "rows op, split per key tile")


@pytest.mark.parametrize("G,gamma,s", [(4, 16, 1024), (4, 32, 1024), (4, 128, 1536), (4, 8, 1000),
                                       (8, 64, 1024), (8, 16, 1024), (8, 32, 1280), (8, 128, 1536)])
def test_fused_delta_all_strides_and_groups(G, gamma, s):
    """Every fused-delta arrangement: anchors inside one warp's rows (gamma <= R),
    in tile A for tile B (gamma = 2R), and over several consecutive jobs of one
    CTA (gamma > 2R).  The fp32 telemetry the windowed launch writes must be the
    oracle's dense minus sparse row at every anchor, and the output must match."""
    Hkv, d, window, sink = 2, 128, 320, 48
    H = G * Hkv
    q, k, v = make_inputs(s, H, Hkv, d, seed=100 + G + gamma)
    out, delta = _run(q, k, v, gamma=gamma, window=window, sink=sink, return_anchor_delta=True, check=True)
    anchors, _, _ = orc.anchor_layout(s, gamma)
    sc = d ** -0.5
    qf, kf, vf = q.float(), k.float(), v.float()
    ref = orc.dense_rows(qf, kf, vf, anchors, sc) - orc.sparse_rows(qf, kf, vf, anchors, window, sink, sc)
    assert_close(delta.cpu(), ref, f"fused delta G={G} gamma={gamma}")
    assert_close(out.cpu(), _oracle_full(q, k, v, gamma, window, sink), f"fused output G={G} gamma={gamma}")
