"""Deferred folding (window > 1, the reference's deferred hook mode): tiles kept
and folded in one launch (ifk_tsqr_fold_segments) give the factors of the
streaming folds.  Both are held
to the fp64 damped factor of all rows; the deferred schedule must be as
accurate as the streaming one (fp32 mode to 2e-5, bf16 mode within the bf16
mode's own error)."""
import math

import numpy as np
import pytest
import torch

from oracle import ifk_oracle as ora
from ifkfac_b200 import _lib
from ifkfac_b200.engine import LayerCurvature

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prec,tol", [(_lib.PREC_FP32, 2e-5), (_lib.PREC_BF16, 2e-2)])
def test_deferred_window_matches_streaming(prec, tol):
    n, tile, ntile = 192, 96, 5
    g = torch.Generator(device="cuda").manual_seed(3)
    s = torch.exp(torch.rand(n, generator=g, device="cuda") * math.log(100.0))
    X = torch.randn(tile * ntile, n, generator=g, device="cuda") * s
    D = torch.randn(tile * ntile, n, generator=g, device="cuda") * s
    dt = torch.float32 if prec == _lib.PREC_FP32 else torch.bfloat16
    X, D = X.to(dt), D.to(dt)
    out = []
    for window in (1, 3):
        lc = LayerCurvature(n, n, "cuda", prec, torch.float32, tile, window=window)
        for t in range(ntile):
            lc.fold(X[t * tile:(t + 1) * tile], D[t * tile:(t + 1) * tile])
        assert lc.refresh(1e-2)
        out.append((lc.RX.double().cpu().numpy(), lc.RG.double().cpu().numpy(), lc.fx.rows_seen))
    (ax, ag, na), (bx, bg, nb) = out
    assert na == nb == tile * ntile

    def truth(M):
        R = ora.positive_diagonal_R(ora._qr_r(M.double().cpu().numpy()))
        return ora.positive_diagonal_R(ora._qr_r(np.concatenate([R / math.sqrt(M.shape[0]),
                                                               math.sqrt(1e-2) * np.eye(n)], 0)))

    rel = lambda x, y: np.linalg.norm(x - y) / np.linalg.norm(y)
    for stream, defer, M in ((ax, bx, X), (ag, bg, D)):
        t = truth(M)
        e_s, e_d = rel(stream, t), rel(defer, t)
        assert e_d < tol and e_d <= 1.5 * e_s + tol / 10, (e_d, e_s)
