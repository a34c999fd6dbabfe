"""GPU parity of the fp32 path (IFK_PREC_FP32) against the CPU oracle and the golden vectors.

Tolerance: relative Frobenius error <= 1e-5 of the natural gradient (the fp32
bound of the task), and the same bound on R factors; R is compared directly
because both sides use the non-negative-diagonal convention.
"""
import math

import numpy as np
import pytest
import torch

from oracle import ifk_oracle as O
from tests.golden_io import load, rel

pytestmark = pytest.mark.gpu
DEV = "cuda"
FP32 = 1  # IFK_PREC_FP32


def _t(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def _scaled(rng, p, n, dtype=np.float32):
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    return (rng.standard_normal((p, n)) * s).astype(dtype)


def test_streaming_golden_sequence():
    from ifkfac_b200 import triangular as T
    g = load("streaming_tsqr")
    R = None
    total = 0
    for i, r in enumerate(g["f32_rows"]):
        R = T.streaming_tsqr_update(R, _t(g[f"f32_chunk{i}"]), prec=FP32)
        total += int(r)
        ref = g[f"f32_R{i}"]
        assert tuple(R.shape) == ref.shape
        assert rel(R.cpu().numpy(), ref) < 1e-5, (i, rel(R.cpu().numpy(), ref))
    F = T.finalize_R(R / math.sqrt(total), 1e-2, prec=FP32)
    assert rel(F.cpu().numpy(), g["f32_final"]) < 1e-5


@pytest.mark.parametrize("n,rows", [(10, [7, 30]), (64, [64, 64, 5]), (100, [300]),
                                    (257, [100, 300, 17]), (512, [256, 1024])])
def test_fold_matches_oracle(n, rows):
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(n)
    R = None
    Ro = None
    for p in rows:
        X = _scaled(rng, p, n)
        R = T.streaming_tsqr_update(R, _t(X), prec=FP32)
        Ro = O.streaming_tsqr_update(Ro, X)
        assert tuple(R.shape) == Ro.shape
        assert rel(R.cpu().numpy(), Ro) < 1e-5


def test_bf16_chunk_fp32_mode():
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(1)
    X = O.bf16_round(_scaled(rng, 700, 200))
    R = T.streaming_tsqr_update(None, _t(X, torch.bfloat16), prec=FP32)
    assert rel(R.cpu().numpy(), O.streaming_tsqr_update(None, X)) < 1e-5


def test_finalize_and_factor_scaling():
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(2)
    X = _scaled(rng, 600, 192)
    rf = T.RunningFactor(192, DEV, prec=FP32)
    rf.fold(_t(X[:150]))
    assert rf.damped(1e-2) is None          # still trapezoidal: the reference skips the layer
    rf.fold(_t(X[150:]))
    F = rf.damped(1e-2).cpu().numpy()
    Fo = O.get_factor(O.streaming_tsqr_update(None, X), 600, 1e-2)
    assert rel(F, Fo) < 1e-5
    Fb = rf.damped(1e-2, out_dtype=torch.bfloat16)
    assert Fb.dtype == torch.bfloat16
    assert rel(Fb.float().cpu().numpy(), O.bf16_round(Fo)) < 1e-2


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_apply_vered_golden(tag):
    from ifkfac_b200 import triangular as T
    g = load("apply_vered")
    dt = torch.bfloat16 if tag == "bf16" else torch.float32
    nat = T.apply_vered(_t(g["f32_gW"]), _t(g[f"{tag}_RX"], dt), _t(g[f"{tag}_RG"], dt), prec=FP32)
    assert rel(nat.cpu().numpy(), g[f"{tag}_nat"]) < 1e-5
    natb = T.apply_vered_bias(_t(g["f32_gb"]), _t(g[f"{tag}_RG"], dt), prec=FP32)
    assert rel(natb.cpu().numpy(), g[f"{tag}_natb"]) < 1e-5


@pytest.mark.parametrize("n_out,n_in", [(24, 40), (130, 70), (256, 512)])
def test_natgrad_matches_oracle(n_out, n_in):
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(n_out + n_in)
    RX = O.get_factor(O.streaming_tsqr_update(None, _scaled(rng, 2 * n_in, n_in)), 2 * n_in, 1e-2)
    RG = O.get_factor(O.streaming_tsqr_update(None, _scaled(rng, 2 * n_out, n_out)), 2 * n_out, 1e-2)
    gW = (rng.standard_normal((n_out, n_in)) * 1e-2).astype(np.float32)
    nat = T.apply_vered(_t(gW), _t(RX), _t(RG), prec=FP32).cpu().numpy()
    assert rel(nat, O.apply_vered(gW, RX, RG)) < 1e-5


def test_update_epilogue_matches_oracle():
    from ifkfac_b200 import triangular as T
    rng = np.random.default_rng(3)
    W = rng.standard_normal((33, 17)).astype(np.float32)
    for clip, mom, wd in [(None, 0.9, 0.0), (0.5, 0.9, 0.1), (None, 0.0, 0.01)]:
        Wd = _t(W)
        bufd = torch.zeros_like(Wd)
        Wo, bo = W.copy(), None
        for it in range(3):
            nat = (rng.standard_normal(W.shape) * 0.3).astype(np.float32)
            T.precond_update_(Wd, bufd if mom > 0 else None, _t(nat), 0.1, mom, wd, clip, it == 0)
            Wo, bo = O.precond_update(Wo, bo, nat, 0.1, mom, wd, clip)
        assert rel(Wd.cpu().numpy(), Wo) < 1e-6
        if mom > 0:
            assert rel(bufd.cpu().numpy(), bo) < 1e-6
