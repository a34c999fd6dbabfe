"""ifk_rtree_merge: the reference's tsqr merge tree (ifkfac/triangular.py:207-220)
on factors one process holds, each round in one launch, against the QR of all
rows (the oracle) and against the pairwise Python tree on the same kernels."""
import math

import numpy as np
import pytest

from ifkfac_b200 import _lib
from oracle import ifk_oracle as O
from tests.golden_io import rel

pytestmark = pytest.mark.gpu


def _blocks(n, per, seed):
    rng = np.random.default_rng(seed)
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    return [O.bf16_round((rng.standard_normal((p, n)) * s).astype(np.float32)) for p in per]


@pytest.mark.parametrize("prec,tol", [(_lib.PREC_FP32, 1e-5), (_lib.PREC_BF16, 1e-2)])
@pytest.mark.parametrize("n,per", [(96, [200, 60, 0, 150, 300]), (520, [600, 333, 1024])])
def test_rtree_merge_matches_qr_of_all_rows(prec, tol, n, per):
    import torch
    from ifkfac_b200 import distributed as D
    blocks = _blocks(n, per, n + len(per))
    factors, rows = [], []
    for X in blocks:
        R = np.zeros((n, n), np.float32)
        if X.shape[0]:
            r = O.positive_diagonal_R(O._qr_r(X))
            R[: r.shape[0]] = r
        factors.append(torch.from_numpy(R).cuda())
        rows.append(min(n, X.shape[0]))
    pyf = [f.clone() for f in factors]
    got_rows = D.tree_merge_device(factors, rows, prec)
    torch.cuda.synchronize()
    want = O.positive_diagonal_R(O._qr_r(np.concatenate(blocks, 0)))
    assert got_rows == min(n, sum(rows))
    e = rel(factors[0].cpu().numpy()[: want.shape[0]], want)
    assert e < tol, e
    assert np.all(np.diagonal(factors[0].cpu().numpy())[:got_rows] >= 0)
    # the same tree pair by pair (one fold call per merge) gives the same factor
    out, r2 = D.tree_merge(pyf, rows, lambda a, ra, b, rb: D.fold_merge(a, ra, b, rb, prec))
    torch.cuda.synchronize()
    assert r2 == got_rows
    assert np.array_equal(out.cpu().numpy(), factors[0].cpu().numpy())
