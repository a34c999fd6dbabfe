"""Pin the CPU oracle against golden vectors produced by the reference itself.

Each test runs the oracle restatement on the inputs saved by
tests/golden/make_golden.py and compares with the reference's outputs.
Tolerances: float64 to 1e-11 relative (LAPACK implementations differ only in
rounding), float32 to 2e-5, bf16 restatement bit-exact.
"""
import math

import numpy as np
import pytest

from oracle import bf16_oracle as B
from oracle import ifk_oracle as O
from tests.golden_io import load, rel

TOL = {"f64": 1e-11, "f32": 2e-5}


@pytest.mark.parametrize("tag", ["f64", "f32"])
def test_streaming_tsqr_matches_reference(tag):
    g = load("streaming_tsqr")
    R = None
    total = 0
    for i, r in enumerate(g[f"{tag}_rows"]):
        R = O.streaming_tsqr_update(R, g[f"{tag}_chunk{i}"])
        total += int(r)
        ref = g[f"{tag}_R{i}"]
        assert R.shape == ref.shape            # trapezoid (20x48) until 48 rows seen
        assert np.all(np.diagonal(R) >= 0)     # positive-diagonal convention
        assert rel(R, ref) < TOL[tag], (i, rel(R, ref))
    Rs = O.scale_rows(R, total)
    assert rel(O.finalize_R(Rs, 1e-2), g[f"{tag}_final"]) < TOL[tag]
    assert rel(O.finalize_R(Rs, 1e-3), g[f"{tag}_final_l3"]) < TOL[tag]


@pytest.mark.parametrize("tag", ["f64", "f32"])
def test_apply_vered_matches_reference(tag):
    g = load("apply_vered")
    nat = O.apply_vered(g[f"{tag}_gW"], g[f"{tag}_RX"], g[f"{tag}_RG"])
    assert rel(nat, g[f"{tag}_nat"]) < TOL[tag] * 10
    natb = O.apply_vered_bias(g[f"{tag}_gb"], g[f"{tag}_RG"])
    assert rel(natb, g[f"{tag}_natb"]) < TOL[tag] * 10


def test_apply_vered_bf16_storage_and_batched():
    g = load("apply_vered")
    nat = O.apply_vered(g["f32_gW"], g["bf16_RX"], g["bf16_RG"], r_is_bf16=True)
    assert rel(nat, g["bf16_nat"]) < 2e-5
    assert rel(O.apply_vered_bias(g["f32_gb"], g["bf16_RG"]), g["bf16_natb"]) < 2e-5
    for b in range(g["batched_gW"].shape[0]):
        nb = O.apply_vered(g["batched_gW"][b], g["f32_RX"], g["f32_RG"])
        assert rel(nb, g["batched_nat"][b]) < 2e-4


def test_batched_fold_and_tree_match_reference():
    g = load("batched_tree")
    out = O.batched_streaming_tsqr_update(g["running"], g["chunks"])
    assert rel(out, g["out"]) < 2e-5
    assert rel(O.tsqr(g["M"], 64), g["tree64"]) < 1e-11
    assert rel(O.tsqr(g["M"], 512), g["tree200"]) < 1e-11


def test_bf16_linalg_restatement_bit_exact():
    g = load("bf16_linalg")
    for tag in ("a", "b"):
        R = B.block_householder_qr_bf16(g[f"qr_{tag}_A"], int(g[f"qr_{tag}_bs"]))
        assert np.array_equal(R, g[f"qr_{tag}_R"]), (tag, rel(R, g[f"qr_{tag}_R"]))
    assert np.array_equal(B.solve_triangular_bf16(g["tri_R"], g["tri_B"], True), g["tri_up"])
    assert np.array_equal(B.solve_triangular_bf16(np.ascontiguousarray(g["tri_R"].T), g["tri_B"], False),
                          g["tri_lo"])
    lam = float(g["comp_lam"])
    RX, RG = B.bf16_factor(g["comp_X"], lam), B.bf16_factor(g["comp_D"], lam)
    assert np.array_equal(O.bf16_round(RX), g["comp_RX"])
    assert np.array_equal(O.bf16_round(RG), g["comp_RG"])
    assert np.array_equal(B.bf16_natgrad(g["comp_gW"], g["comp_RX"], g["comp_RG"]), g["comp_nat"])


def test_hooks_factors_match_oracle_composition():
    """3-D inputs (max_seq_rows=0) are flattened to rows; augment_bias appends a ones column;
    get_factors = finalize_R(R/sqrt(rows))."""
    import torch
    import torch.nn as nn
    g = load("hooks_seq_bias")
    torch.manual_seed(2)
    model = nn.Sequential(nn.Linear(12, 20), nn.GELU(), nn.Linear(20, 6))
    model.load_state_dict({k[5:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("init_")})
    layers = [model[0], model[2]]
    acts = {0: [], 1: []}
    grads = {0: [], 1: []}
    hs = []
    for i, m in enumerate(layers):
        hs.append(m.register_forward_hook(lambda mod, inp, out, i=i: acts[i].append(inp[0].detach())))
        hs.append(m.register_full_backward_hook(lambda mod, gi, go, i=i: grads[i].append(go[0].detach())))
    for k in range(3):
        model(torch.from_numpy(g[f"x{k}"])).square().sum().backward()
    for h in hs:
        h.remove()
    for i in range(2):
        RX = RG = None
        rx = rg = 0
        for a in acts[i]:
            a = a.reshape(-1, a.shape[-1]).numpy()
            a = np.concatenate([a, np.ones((a.shape[0], 1), a.dtype)], 1)
            RX = O.streaming_tsqr_update(RX, a)
            rx += a.shape[0]
        for d in grads[i]:
            d = d.reshape(-1, d.shape[-1]).numpy()
            RG = O.streaming_tsqr_update(RG, d)
            rg += d.shape[0]
        assert [rx, rg] == list(g[f"rows{i}"])
        assert rel(RX, g[f"rawRX{i}"]) < 2e-5 and rel(RG, g[f"rawRG{i}"]) < 2e-5
        assert rel(O.get_factor(RX, rx, 1e-3), g[f"RX{i}"]) < 2e-5
        assert rel(O.get_factor(RG, rg, 1e-3), g[f"RG{i}"]) < 2e-5


def test_refresh_schedule():
    assert [O.should_refresh(s, 1) for s in range(1, 4)] == [True] * 3
    assert [s for s in range(1, 31) if O.should_refresh(s, 10)] == [10, 20, 30]
    assert [s for s in range(1, 8) if O.should_refresh(s, 3)] == [3, 6]


def test_precond_update_rules():
    rng = np.random.default_rng(0)
    W = rng.standard_normal((4, 3)).astype(np.float32)
    g = rng.standard_normal((4, 3)).astype(np.float32)
    W1, b1 = O.precond_update(W, None, g, lr=0.1, momentum=0.9, weight_decay=0.0, grad_clip=None)
    assert np.allclose(b1, g) and np.allclose(W1, W - 0.1 * g)
    W2, b2 = O.precond_update(W1, b1, g, lr=0.1, momentum=0.9, weight_decay=0.5, grad_clip=None)
    assert np.allclose(b2, 0.9 * g + g)
    assert np.allclose(W2, W1 * (1 - 0.05) - 0.1 * b2, atol=1e-6)
    W3, _ = O.precond_update(W, None, g * 100, lr=1.0, momentum=0.0, weight_decay=0.0, grad_clip=1.0)
    assert abs(np.linalg.norm(W - W3) - 1.0) < 1e-5


def test_ema_blend_restatement_matches_reference():
    """oracle.ema_blend reproduces the reference's blended factors: the step-4 refresh
    of a gamma = 0.4 run blends the step-2 factors with the step-4 ones (those of the
    gamma = 0 run, identical up to step 3)."""
    z = load("ema_blend")
    for i in range(2):
        for f in ("RX", "RG"):
            old, new = z[f"ema_s2_{f}{i}"].astype(np.float64), z[f"plain_s4_{f}{i}"].astype(np.float64)
            assert np.array_equal(z[f"ema_s2_{f}{i}"], z[f"plain_s2_{f}{i}"])
            got = O.ema_blend(old, new, 0.4)
            ref = z[f"ema_s4_{f}{i}"].astype(np.float64)
            assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-5


def test_laplace_draw_restatement_matches_reference():
    """LaplacePosterior.sample_in_place (ifkfac/laplace.py:127-146) from EVD
    factors of svd(R): the restated draw gives the reference's weights, and the
    triangular form (posterior_factor / posterior_sample) has the same posterior
    precision P = U diag(sqrt(N) d + sqrt(lambda)) U^T, so the same distribution."""
    g = load("laplace")
    N, lam = int(g["N"]), float(g["lam"])
    for i in range(2):
        W = g[f"Wmap{i}"] + O.laplace_sample_evd(g[f"U_A{i}"], g[f"d_A{i}"], g[f"U_G{i}"], g[f"d_G{i}"],
                                                 g[f"xi{i}"], N, lam)
        assert rel(W, g[f"Wsample{i}"]) < 1e-6
        for tag in ("A", "G"):
            R = g[f"R_{tag}{i}"].astype(np.float64)
            C = O.posterior_factor(R, N, lam)
            U, d = g[f"U_{tag}{i}"].astype(np.float64), g[f"d_{tag}{i}"].astype(np.float64)
            P = U @ np.diag(math.sqrt(N) * d + math.sqrt(lam)) @ U.T
            assert rel(C.T @ C, P) < 1e-5
        # same covariance per side: (C^T C)^-1 = U diag(s^2) U^T
        for tag in ("A", "G"):
            C = O.posterior_factor(g[f"R_{tag}{i}"].astype(np.float64), N, lam)
            U, d = g[f"U_{tag}{i}"].astype(np.float64), g[f"d_{tag}{i}"].astype(np.float64)
            S = U @ np.diag(O.laplace_scales(d, N, lam) ** 2) @ U.T
            assert rel(np.linalg.inv(C.T @ C), S) < 1e-5
