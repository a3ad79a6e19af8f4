"""Pin the CPU oracle to the reference's own outputs (golden fixtures made by
``tests/golden/make_golden.py`` from the reference's CPU-runnable code)."""

import json
import os

import numpy as np
import pytest
import torch

from delta_attention_b200.synthetic import make_inputs, tensor_digest
from oracle import delta_oracle as orc
from tests.golden.make_golden import DECODE_SHAPE, FLEX_CASES, decode_inputs

FLEX_NAMES = [n for n in FLEX_CASES if n != "flex_config1"]


def _load(golden_dir, name):
    z = np.load(os.path.join(golden_dir, f"{name}.npz"))
    return z, json.loads(str(z["meta"]))


def _inputs(meta):
    theta = None if meta["rope_theta"] < 0 else meta["rope_theta"]
    q, k, v = make_inputs(meta["s"], meta["H"], meta["Hkv"], meta["d"], seed=meta["seed"],
                          rope_theta=theta, dtype=torch.bfloat16)
    assert tensor_digest(q, k, v) == meta["digest"], "synthetic input generator drifted"
    return q.float(), k.float(), v.float()


@pytest.mark.parametrize("name", FLEX_NAMES + [pytest.param("flex_config1", marks=pytest.mark.slow)])
def test_oracle_matches_reference_flex(golden_dir, name):
    z, meta = _load(golden_dir, name)
    q, k, v = _inputs(meta)
    rows = torch.from_numpy(z["rows"]).long()
    ref = torch.from_numpy(z["out"]).double()
    got = orc.delta_forward_rows(q, k, v, rows, meta["gamma"], meta["window"], meta["sink"])[0]
    err = (got - ref).abs().max().item()
    assert err < 2e-5, f"{name}: oracle vs reference max abs err {err}"
    if meta["s"] <= 1024:
        full = orc.delta_forward(q, k, v, meta["gamma"], meta["window"], meta["sink"])[0]
        cs = torch.from_numpy(z["checksum"])
        assert (full.sum(0) - cs).abs().max().item() < 1e-3
        assert (full[rows] - got).abs().max().item() < 1e-10


def test_oracle_config1_checksum_rows(golden_dir):
    """Config 1 (s=4096, 32/8 heads): sampled rows only (full oracle ~1 min)."""
    z, meta = _load(golden_dir, "flex_config1")
    q, k, v = _inputs(meta)
    rows = torch.from_numpy(z["rows"]).long()[:12]
    ref = torch.from_numpy(z["out"][:12]).double()
    got = orc.delta_forward_rows(q, k, v, rows, meta["gamma"], meta["window"], meta["sink"])[0]
    assert (got - ref).abs().max().item() < 2e-5


def test_oracle_variable_stride(golden_dir):
    z = np.load(os.path.join(golden_dir, "stride_variable.npz"))
    meta = json.loads(str(z["meta"]))
    got = orc.apply_delta_variable(torch.from_numpy(z["sparse"]), torch.from_numpy(z["dense_sel"]),
                                   torch.from_numpy(z["idx"]), meta["s_p"])
    assert torch.equal(got, torch.from_numpy(z["corrected"]))


def test_oracle_layout_bit_exact(golden_dir):
    z = np.load(os.path.join(golden_dir, "stride_variable.npz"))
    meta = json.loads(str(z["meta"]))
    for L in meta["layouts"]:
        a, t, s_p = orc.anchor_layout(L["s"], L["gamma"])
        assert a.numel() == L["n_anchor"] and t.numel() == L["n_tail"]
        assert int(a.sum()) == L["anchor_sum"]
        if t.numel():
            assert int(t[0]) == L["first_tail"]
        assert orc.uniform_effective_sparsity(L["s"], L["gamma"], 2048, 128) == pytest.approx(L["eff"], abs=1e-12)


def test_oracle_decode_matches_reference(golden_dir):
    z, meta = _load(golden_dir, "decode_reference")
    qs, k, v = decode_inputs()
    assert tensor_digest(torch.stack(qs), k, v) == meta["digest"]
    sc = meta["scaling"]
    for policy in ("fixed", "drift", "drift_rel"):
        st = orc.OracleDecodeState()
        cfg = meta[policy]
        ref = torch.from_numpy(z[f"out_{policy}"])
        for t in range(meta["steps"]):
            out, anchor = orc.delta_decode_step(
                st, qs[t], k, v, window=meta["window"], sink=meta["sink"], scaling=sc,
                gamma_dec=cfg["gamma_dec"], refresh_policy=policy,
                drift_threshold=cfg.get("drift_threshold", 0.95), drift_k=cfg.get("drift_k", 2.0),
                gamma_dec_max=128)
            assert anchor == cfg["anchors"][t], (policy, t)
            assert (out - ref[t].double()).abs().max().item() < 2e-5, (policy, t)
    sp = orc.sparse_decode(qs[0], k, v, meta["window"], meta["sink"], sc)
    assert (sp - torch.from_numpy(z["out_sparse"]).double()).abs().max().item() < 2e-5


def test_oracle_gradients_match_reference_finite_differences(golden_dir):
    """The oracle's training forward, differentiated by autograd, against central
    finite differences of the reference's own ``delta_forward_train`` along the
    same seeded directions (``tests/golden/train_fd.json``)."""
    from tests.golden.make_golden import TRAIN_FD_CASES, train_fd_tensors

    with open(os.path.join(golden_dir, "train_fd.json")) as f:
        rec = json.load(f)
    for name, case in TRAIN_FD_CASES.items():
        want = rec["cases"][name]["directional_derivatives"]
        assert rec["cases"][name]["case"] == list(case)
        s, H, Hkv, d, gamma, window, sink, seed = case
        for i, fd in enumerate(want):
            (q, k, v), w, dirs = train_fd_tensors(case, i)
            q, k, v = (t.clone().requires_grad_(True) for t in (q, k, v))
            out = orc.delta_forward_train(q, k, v, gamma, window, sink)
            (out * w).sum().backward()
            got = sum(float((t.grad * dt).sum()) for t, dt in zip((q, k, v), dirs))
            assert abs(got - fd) <= 1e-6 * max(1.0, abs(fd)), f"{name} dir {i}: autograd {got} vs reference fd {fd}"


def test_oracle_training_arms():
    """detach_delta keeps the forward and removes the delta path's gradient;
    delta_grad_scale interpolates (flex_delta.py:189-192)."""
    torch.manual_seed(3)
    s, H, Hkv, d = 512, 4, 1, 32
    q0, k0, v0 = (torch.randn(1, h, s, d, dtype=torch.float64) for h in (H, Hkv, Hkv))
    w = torch.randn(1, s, H, d, dtype=torch.float64)

    def grads(**kw):
        q, k, v = (t.clone().requires_grad_(True) for t in (q0, k0, v0))
        out = orc.delta_forward_train(q, k, v, 64, 128, 32, **kw)
        (out * w).sum().backward()
        return out.detach(), q.grad, k.grad, v.grad

    full, det, half = grads(), grads(detach_delta=True), grads(delta_grad_scale=0.5)
    assert torch.equal(full[0], det[0]) and torch.equal(full[0], half[0])
    for a, b, c in zip(full[1:], det[1:], half[1:]):
        assert (a - b).norm() > 1e-3 * a.norm()
        assert torch.allclose(c, 0.5 * (a + b), atol=1e-10)
