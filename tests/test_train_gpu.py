"""Training path on the GPU: the forward's log-sum-exp outputs and the
backward kernels (dta_backward) against the oracle's autograd gradients
(oracle.delta_forward_train, pinned to the reference by finite differences in
tests/test_oracle_golden.py), plus the reference's T14 checks
(tests/test_flex_delta.py:88-160).

Gradient tolerance: P and dS enter the tensor cores as bf16 and the gradients
leave as bf16, so each gradient tensor is compared normwise: relative error
||got - ref|| / ||ref|| <= GRAD_REL and cosine >= GRAD_COS, per head for dq
(per KV head for dk, dv) as well as overall."""

import math

import pytest
import torch

from delta_attention_b200 import ops, train
from delta_attention_b200.synthetic import make_inputs
from oracle import delta_oracle as orc

pytestmark = pytest.mark.gpu

GRAD_REL = 1.5e-2
GRAD_COS = 0.9998
LSE_ABS = 2e-3  # base-2 log-sum-exp, absolute


def _oracle_lse2(q, k, rows, keep_fn, scaling):
    """log2 of the softmax denominator of scaled scores, [b, H, n] (float64)."""
    b, H, s, d = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    qq = q[:, :, rows].double().reshape(b, Hkv, G, rows.numel(), d)
    kk = k.double().unsqueeze(2)
    sc = torch.matmul(qq, kk.transpose(-1, -2)) * scaling  # [b, Hkv, G, n, s]
    keep = keep_fn(rows[:, None], torch.arange(s)[None, :])
    sc = sc.masked_fill(~keep, float("-inf"))
    return (torch.logsumexp(sc, dim=-1) / math.log(2.0)).reshape(b, H, rows.numel())


LSE_CASES = [
    # s, H, Hkv, d, gamma, window, sink
    (1024, 8, 2, 128, 64, 256, 64),     # 4 heads per group, pair-fused delta
    (1024, 8, 1, 128, 128, 192, 128),   # 8 heads per group
    (768, 4, 4, 64, 64, 128, 32),       # 1 head per group (delta kernel path)
    (768, 4, 2, 64, 32, 256, 64),       # 2 heads per group
]


@pytest.mark.parametrize("case", LSE_CASES, ids=lambda c: "s{}_h{}_{}_d{}_g{}".format(*c[:5]))
def test_prefill_lse_outputs_match_oracle(case):
    s, H, Hkv, d, gamma, window, sink = case
    q, k, v = make_inputs(s, H, Hkv, d, seed=11, rope_theta=500000.0, dtype=torch.bfloat16)
    anchors, tail, s_p = train.anchor_layout(s, gamma)
    sel = torch.cat((anchors, tail))
    lse_sp = torch.full((1, H, s), float("nan"), dtype=torch.float32, device="cuda")
    lse_dn = torch.full((1, H, sel.numel()), float("nan"), dtype=torch.float32, device="cuda")
    ops.prefill(q.cuda(), k.cuda(), v.cuda(), gamma=gamma, window=window, sink=sink, return_anchor_delta=True,
                lse_sparse=lse_sp, lse_dense=lse_dn, check=True)
    scaling = d ** -0.5
    want_sp = _oracle_lse2(q, k, torch.arange(s_p), lambda r, c: orc.sparse_keep(r, c, window, sink), scaling)
    want_dn = _oracle_lse2(q, k, sel, lambda r, c: c <= r, scaling)
    got_sp = lse_sp[:, :, :s_p].double().cpu()
    got_dn = lse_dn.double().cpu()
    assert torch.isfinite(got_sp).all() and torch.isfinite(got_dn).all()
    e1 = (got_sp - want_sp).abs().max().item()
    e2 = (got_dn - want_dn).abs().max().item()
    assert e1 <= LSE_ABS and e2 <= LSE_ABS, f"lse max abs err sparse {e1:.2e} dense {e2:.2e}"


def _grad_check(got, ref, what, per_dim=1):
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    assert torch.isfinite(got).all(), f"{what}: non-finite gradient"
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    g = got.transpose(0, per_dim).reshape(got.shape[per_dim], -1)
    r = ref.transpose(0, per_dim).reshape(ref.shape[per_dim], -1)
    cos_h = torch.nn.functional.cosine_similarity(g, r, dim=1).min().item()
    print(f"{what}: rel {rel:.3e} cos {cos:.6f} min per-head cos {cos_h:.6f}")
    assert rel <= GRAD_REL, f"{what}: normwise relative error {rel:.3e} > {GRAD_REL}"
    assert cos >= GRAD_COS and cos_h >= GRAD_COS, f"{what}: cosine {cos:.6f} / per head {cos_h:.6f} < {GRAD_COS}"


BWD_CASES = [
    # s, H, Hkv, d, gamma, window, sink, detach, scale
    (512, 4, 1, 64, 64, 128, 32, False, 1.0),
    (768, 4, 2, 64, 32, 256, 64, False, 1.0),
    (1024, 8, 2, 128, 128, 192, 128, False, 1.0),
    (1024, 8, 1, 128, 64, 256, 64, False, 1.0),      # 8 heads per group (R = 16)
    (640, 4, 4, 128, 64, 128, 0, False, 1.0),        # 1 head per group (R = 128), no sink
    (1088, 4, 1, 128, 64, 320, 200, False, 1.0),     # partial key tile, sink not a tile multiple
    (1024, 8, 2, 128, 64, 256, 64, True, 1.0),       # detach_delta arm
    (1024, 8, 2, 128, 64, 256, 64, False, 0.125),    # delta_grad_scale arm
]


@pytest.mark.parametrize("case", BWD_CASES, ids=lambda c: "s{}_h{}_{}_d{}_g{}_w{}_s{}_{}_{}".format(*c))
def test_backward_matches_oracle(case):
    s, H, Hkv, d, gamma, window, sink, detach, scale = case
    q, k, v = make_inputs(s, H, Hkv, d, seed=5, rope_theta=500000.0, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(17)
    gout = torch.randn(1, s, H, d, generator=gen).bfloat16()
    # oracle: float64 autograd on the same bf16 values
    qo, ko, vo = (t.double().requires_grad_(True) for t in (q, k, v))
    ref_out = orc.delta_forward_train(qo, ko, vo, gamma, window, sink, detach_delta=detach, delta_grad_scale=scale)
    (ref_out * gout.double()).sum().backward()
    # kernels
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    out = train.delta_forward_train(qc, kc, vc, gamma, window, sink, detach_delta=detach, delta_grad_scale=scale)
    out.backward(gout.cuda())
    ops.check_errors()
    _grad_check(out, ref_out, "out", per_dim=2)
    _grad_check(qc.grad, qo.grad, "dq")
    _grad_check(kc.grad, ko.grad, "dk")
    _grad_check(vc.grad, vo.grad, "dv")


def test_backward_config1_matches_oracle():
    """The benchmark matrix's config 1 (s=4096, 32/8 heads, d=128, W=1024, S=64,
    gamma=64; the reference's CPU-runnable training shape): every gradient
    against the oracle's float64 autograd on the same bf16 inputs."""
    s, H, Hkv, d, gamma, window, sink = 4096, 32, 8, 128, 64, 1024, 64
    q, k, v = make_inputs(s, H, Hkv, d, seed=0, rope_theta=500000.0, dtype=torch.bfloat16)
    gout = torch.randn(1, s, H, d, generator=torch.Generator().manual_seed(1)).bfloat16()
    qo, ko, vo = (t.double().requires_grad_(True) for t in (q, k, v))
    (orc.delta_forward_train(qo, ko, vo, gamma, window, sink) * gout.double()).sum().backward()
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    train.delta_forward_train(qc, kc, vc, gamma, window, sink).backward(gout.cuda())
    ops.check_errors()
    _grad_check(qc.grad, qo.grad, "config1 dq")
    _grad_check(kc.grad, ko.grad, "config1 dk")
    _grad_check(vc.grad, vo.grad, "config1 dv")


def _t14_inputs(seed=0):
    torch.manual_seed(seed)
    q = torch.randn(1, 32, 4096, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    return q, k, v


def test_t14_gradient_sanity():
    """Gradients flow and are finite; the anchor-row gradient ratio is a finite
    positive metric (tests/test_flex_delta.py:88-112)."""
    q, k, v = _t14_inputs()
    out = train.delta_forward_train(q, k, v, gamma=64, window=2048)
    out.float().pow(2).mean().backward()
    for name, t in (("q", q), ("k", k), ("v", v)):
        assert t.grad is not None and torch.isfinite(t.grad.float()).all() and t.grad.abs().sum() > 0, name
    ratio = train.anchor_grad_ratio(q.grad, 64)
    assert 0.0 < ratio < float("inf")


def test_t14_delta_path_gradient():
    """Detaching the reused delta changes the gradients measurably
    (tests/test_flex_delta.py:115-140)."""

    def grads(detach):
        q, k, v = _t14_inputs()
        out = train.delta_forward_train(q, k, v, gamma=64, window=2048, detach_delta=detach)
        out.float().pow(2).mean().backward()
        return q.grad.clone(), k.grad.clone(), v.grad.clone()

    full, det = grads(False), grads(True)
    rel = [((a - b).float().norm() / b.float().norm().clamp_min(1e-12)).item() for a, b in zip(full, det)]
    assert max(rel) > 1e-3, rel


def test_t14_detach_delta_ablation():
    """With the delta detached the sparse path's q gradient still flows
    (tests/test_flex_delta.py:143-156)."""
    torch.manual_seed(0)
    q = torch.randn(1, 32, 4096, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16)
    out = train.delta_forward_train(q, k, v, gamma=64, window=2048, detach_delta=True)
    out.float().pow(2).mean().backward()
    assert q.grad is not None and q.grad.abs().sum() > 0


def test_entry_points_from_a_fresh_host_thread():
    """A host thread that has made no CUDA call yet has no current context; the
    entry points make the device's primary context current before encoding
    their TMA descriptors (a driver call that needs one)."""
    import threading

    s, H, Hkv, d, gamma, window, sink = 512, 4, 1, 64, 64, 128, 32
    q, k, v = (t.cuda() for t in make_inputs(s, H, Hkv, d, seed=5, rope_theta=500000.0, dtype=torch.bfloat16))
    _, _, s_p = train.anchor_layout(s, gamma)
    n_sel = s_p // gamma + (s - s_p)
    g = torch.randn(1, s, H, d, device="cuda").bfloat16()
    lse_sp = torch.empty(1, H, s, dtype=torch.float32, device="cuda")
    lse_dn = torch.empty(1, H, n_sel, dtype=torch.float32, device="cuda")
    out, delta = ops.prefill(q, k, v, gamma=gamma, window=window, sink=sink, return_anchor_delta=True,
                             lse_sparse=lse_sp, lse_dense=lse_dn)
    want = ops.backward(q, k, v, out, g, delta, lse_sp, lse_dn, gamma=gamma, window=window, sink=sink)
    torch.cuda.synchronize()
    got, errors = {}, []

    def worker():
        try:
            o, dl = ops.prefill(q, k, v, gamma=gamma, window=window, sink=sink, return_anchor_delta=True,
                                lse_sparse=lse_sp, lse_dense=lse_dn)
            got["out"] = o
            got["grads"] = ops.backward(q, k, v, o, g, dl, lse_sp, lse_dn, gamma=gamma, window=window, sink=sink)
            torch.cuda.synchronize()
        except Exception as e:  # noqa: BLE001 (reported below)
            errors.append(e)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert not errors, errors
    assert torch.equal(got["out"], out)
    for a, b in zip(got["grads"], want):
        assert torch.allclose(a.float(), b.float(), atol=1e-2, rtol=0)
