"""GPU parity of the bf16 tensor-core path (IFK_PREC_BF16).

Reference points:
* the reference's executed path for use_true_bf16 (fp32 QR -> damping fold ->
  bf16 R -> fp32 solves, ifkfac/ifkfac.py:292-294, ifkfac/triangular.py:607-628)
  fed the fp32 upcast of the same bf16 inputs: natural gradient within 2e-2
  relative Frobenius error (the bf16 tolerance);
* the reference's bf16_linalg composition (golden vectors): R factors within
  2e-2 up to row signs.
R factors of the bf16 fold are checked against the fp32 oracle at 1e-2
(bf16 operand rounding, fp32 accumulation and storage).
"""
import math

import numpy as np
import pytest
import torch

from oracle import ifk_oracle as O
from tests.golden_io import load, rel, rel_rowsign

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16, FP32 = 2, 1


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def _scaled_bf16(rng, p, n):
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    return O.bf16_round((rng.standard_normal((p, n)) * s).astype(np.float32))


@pytest.mark.parametrize("n,rows", [(64, [300]), (200, [150, 333]), (512, [256, 1024, 100]),
                                    (700, [2048])])
def test_bf16_fold_matches_oracle(n, rows):
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(n)
    R = None
    Ro = None
    for p in rows:
        X = _scaled_bf16(rng, p, n)
        R = T.streaming_tsqr_update(R, _t(X, torch.bfloat16), prec=BF16)
        Ro = O.streaming_tsqr_update(Ro, X)
        assert tuple(R.shape) == Ro.shape
        e = rel(R.cpu().numpy(), Ro)
        assert e < 1e-2, e
        assert np.all(np.diagonal(R.cpu().numpy()) >= 0)


def test_bf16_factor_and_natgrad_vs_executed_path():
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(7)
    n_in, n_out, p, lam = 384, 256, 1536, 1e-2
    X = _scaled_bf16(rng, p, n_in)
    D = _scaled_bf16(rng, p, n_out)
    gW = (rng.standard_normal((n_out, n_in)) * 1e-2).astype(np.float32)
    fx = T.RunningFactor(n_in, DEV, BF16)
    fd = T.RunningFactor(n_out, DEV, BF16)
    for lo in range(0, p, 512):
        fx.fold(_t(X[lo:lo + 512], torch.bfloat16))
        fd.fold(_t(D[lo:lo + 512], torch.bfloat16))
    RX = fx.damped(lam, out_dtype=torch.bfloat16)
    RG = fd.damped(lam, out_dtype=torch.bfloat16)
    RXo = O.get_factor(O.streaming_tsqr_update(None, X), p, lam)
    RGo = O.get_factor(O.streaming_tsqr_update(None, D), p, lam)
    assert rel(RX.float().cpu().numpy(), RXo) < 1e-2
    assert rel(RG.float().cpu().numpy(), RGo) < 1e-2
    nat_exec = O.apply_vered(gW, O.bf16_round(RXo), O.bf16_round(RGo), r_is_bf16=True)
    for prec in (FP32, BF16):
        nat = T.apply_vered(_t(gW), RX, RG, prec=prec).cpu().numpy()
        assert rel(nat, nat_exec) < 2e-2


def test_bf16_fold_vs_bf16_linalg_golden():
    """R of the reference's bf16_linalg composition (golden) vs the bf16 fold, up to row signs."""
    from ifkfac_b200 import triangular as T
    g = load("bf16_linalg")
    lam = float(g["comp_lam"])
    for key, rkey in (("comp_X", "comp_RX"), ("comp_D", "comp_RG")):
        A = g[key]
        p, n = A.shape
        f = T.RunningFactor(n, DEV, BF16)
        f.fold(_t(A, torch.bfloat16))
        R = f.damped(lam).cpu().numpy()
        assert rel_rowsign(R, g[rkey]) < 2e-2


@pytest.mark.parametrize("n_out,n_in", [(24, 40), (130, 300), (256, 512), (640, 384)])
def test_bf16_natgrad_tensor_core_vs_executed_path(n_out, n_in):
    """Tensor-core trsm on bf16-stored factors vs the reference's fp32 solves on the same factors."""
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(n_out * 7 + n_in)
    RX = O.bf16_round(O.get_factor(O.streaming_tsqr_update(None, _scaled_bf16(rng, 2 * n_in, n_in)),
                                   2 * n_in, 1e-2))
    RG = O.bf16_round(O.get_factor(O.streaming_tsqr_update(None, _scaled_bf16(rng, 2 * n_out, n_out)),
                                   2 * n_out, 1e-2))
    gW = (rng.standard_normal((n_out, n_in)) * 1e-2).astype(np.float32)
    nat = T.apply_vered(_t(gW), _t(RX, torch.bfloat16), _t(RG, torch.bfloat16), prec=BF16)
    e = rel(nat.cpu().numpy(), O.apply_vered(gW, RX, RG, r_is_bf16=True))
    assert e < 5e-3, e


def test_bf16_natgrad_golden():
    from ifkfac_b200 import triangular as T
    g = load("apply_vered")
    nat = T.apply_vered(_t(g["f32_gW"]), _t(g["bf16_RX"], torch.bfloat16), _t(g["bf16_RG"], torch.bfloat16),
                        prec=BF16)
    assert rel(nat.cpu().numpy(), g["bf16_nat"]) < 5e-3


def test_bf16_end_to_end_vs_bf16_linalg_composition():
    """Natural gradient of the full bf16 path vs the reference's bf16_linalg composition.

    The composition's own error against an fp64 truth is 2-3e-2 (its row-by-row
    bf16 solves), so the bound is: no farther from it than its own error plus
    ours, and ours is smaller than its own."""
    from ifkfac_b200 import triangular as T
    g = load("bf16_linalg")
    lam = float(g["comp_lam"])
    X, D, gW = g["comp_X"], g["comp_D"], g["comp_gW"]
    p, n = X.shape
    fs = []
    for A in (X, D):
        f = T.RunningFactor(n, DEV, BF16)
        f.fold(_t(A, torch.bfloat16))
        fs.append(f.damped(lam, out_dtype=torch.bfloat16))
    nat = T.apply_vered(_t(gW), fs[0], fs[1], prec=BF16).cpu().numpy()
    tx = O.get_factor(O.streaming_tsqr_update(None, X.astype(np.float64)), p, lam)
    td = O.get_factor(O.streaming_tsqr_update(None, D.astype(np.float64)), p, lam)
    truth = O.apply_vered(gW.astype(np.float64), tx, td)
    e_ours, e_ref = rel(nat, truth), rel(g["comp_nat"], truth)
    assert e_ours < e_ref
    assert rel(nat, g["comp_nat"]) <= e_ref + e_ours + 1e-6
    assert e_ours < 2e-2


def test_batched_fold_and_finalize_match_single():
    """X and delta folded in one wave schedule give the same factors as separate folds."""
    from ifkfac_b200 import _lib
    from ifkfac_b200.engine import LayerCurvature
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(11)
    n_in, n_out, lam = 320, 200, 1e-2
    X = _scaled_bf16(rng, 900, n_in)
    D = _scaled_bf16(rng, 900, n_out)
    for prec in (FP32, BF16):
        lc = LayerCurvature(n_in, n_out, DEV, prec, torch.float32, 300)
        for lo in range(0, 900, 300):
            lc.fold(_t(X[lo:lo + 300], torch.bfloat16), _t(D[lo:lo + 300], torch.bfloat16))
        assert lc.refresh(lam)
        tol = 1e-5 if prec == FP32 else 1e-2
        assert rel(lc.RX.cpu().numpy(), O.get_factor(O.streaming_tsqr_update(None, X), 900, lam)) < tol
        assert rel(lc.RG.cpu().numpy(), O.get_factor(O.streaming_tsqr_update(None, D), 900, lam)) < tol
