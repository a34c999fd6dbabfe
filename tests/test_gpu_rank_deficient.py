"""Exactly rank-deficient activations: constant columns (GELU outputs pinned at
its minimum round to one bf16 value), duplicated columns and zero columns.  The
running factor then carries zero diagonal entries and later sub-tiles meet
residuals that cancel to zero or to denormals.  The fold must stay finite and
keep R^T R = X^T X (the reference's streaming QR, ifkfac/triangular.py:246-307,
has no rank condition on the chunks)."""
import pytest
import torch

from ifkfac_b200 import _lib
from ifkfac_b200.engine import Factor, fold_segments

pytestmark = pytest.mark.gpu

GELU_MIN_BF16 = -0.169921875  # bf16 of min_x x Phi(x)


def _activations(rows, n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.nn.functional.gelu(torch.randn(rows, n, generator=g, device="cuda") * 0.6)
    for c in range(n // 128, n, n // 5 + 1):  # constant columns, all equal to one another
        x[:, c] = GELU_MIN_BF16
    x[:, n // 3] = x[:, 7]       # a duplicate of an ordinary column
    x[:, n // 2] = 0.0           # a dead column
    x[:, n - 2] = x[:, n - 1]    # a duplicate in the last panel
    return x


@pytest.mark.parametrize("prec,dt,tol", [(_lib.PREC_BF16, torch.bfloat16, 2e-2), (_lib.PREC_FP32, torch.float32, 1e-5)])
@pytest.mark.parametrize("n,rows,chunk", [(768, 4096, 1024), (3072, 1536, 256), (320, 2000, 2000)])
def test_dependent_columns_stay_finite(prec, dt, tol, n, rows, chunk):
    x = _activations(rows, n, n + rows).to(dt)
    f = Factor(n, "cuda", prec)
    for i in range(0, rows, chunk):
        fold_segments((f,), ([x[i:i + chunk]],), None)
    torch.cuda.synchronize()
    assert int(f.status.item()) == 0
    assert torch.isfinite(f.R).all()
    X = x.double()
    G = X.T @ X
    R = f.R.double()
    rel = float((R.T @ R - G).norm() / G.norm())
    assert rel < tol, rel
    # the dependent columns' diagonal entries carry only rounding
    d = R.diagonal().abs()
    assert float(d[n // 2]) < tol * float(d.max())
    assert float(d[n // 3]) < tol * float(d.max())


def test_dependent_columns_damped_refresh():
    """The damped factor of rank-deficient rows is finite with a diagonal >= sqrt(lambda)."""
    n, rows = 768, 3072
    x = _activations(rows, n, 5).to(torch.bfloat16)
    f = Factor(n, "cuda", _lib.PREC_BF16)
    lam = 1e-3
    fold_segments((f,), ([x],), None, ident_tail=[(lam * rows) ** 0.5])
    torch.cuda.synchronize()
    assert int(f.status.item()) == 0
    R = f.R.double() / rows ** 0.5
    assert torch.isfinite(R).all()
    assert float(R.diagonal().abs().min()) >= 0.99 * lam ** 0.5


@pytest.mark.parametrize("prec,dt,tol,tol_trap", [(_lib.PREC_BF16, torch.bfloat16, 2e-2, 5e-2),
                                                   (_lib.PREC_FP32, torch.float32, 1e-5, 1e-5)])
def test_dependent_columns_over_trapezoidal_folds(prec, dt, tol, tol_trap):
    """Folds that end while R is still trapezoidal.  The fp32 fold factors every
    column and is exact at every step (content a zero pivot leaves below row
    rows_R stays in R for the next fold).  The bf16 fold keeps the rank bound: a
    dependent column with a zero or rounding-noise pivot spends its reflector on
    that, and the bound drops one row direction of the sub-tile, so the
    trapezoidal states deviate by up to a few percent (2.2e-2 measured after 200
    rows with 7 of 768 columns dependent); the square factor is back near the
    bf16 level."""
    n, chunk = 768, 200
    x = _activations(1600, n, 17).to(dt)
    f = Factor(n, "cuda", prec)
    for i in range(0, x.shape[0], chunk):
        fold_segments((f,), ([x[i:i + chunk]],), None)
        torch.cuda.synchronize()
        assert int(f.status.item()) == 0
        X = x[: i + chunk].double()
        G = X.T @ X
        R = f.R.double()  # the whole buffer: R^T R holds every row folded so far
        rel = float((R.T @ R - G).norm() / G.norm())
        assert rel < (tol if f.rows_R == n else tol_trap), (i, rel)
    assert f.rows_R == n


@pytest.mark.parametrize("prec,dt,tol", [(_lib.PREC_BF16, torch.bfloat16, 2e-2), (_lib.PREC_FP32, torch.float32, 1e-5)])
def test_merge_of_trapezoidal_factors(prec, dt, tol):
    """fold_merge of two trapezoidal factors of rank-deficient rows (the R-tree's step)."""
    from ifkfac_b200.distributed import fold_merge
    n = 640
    xa = _activations(300, n, 3).to(dt)
    xb = _activations(260, n, 4).to(dt)
    fa, fb = Factor(n, "cuda", prec), Factor(n, "cuda", prec)
    fold_segments((fa,), ([xa],), None)
    fold_segments((fb,), ([xb],), None)
    rows = fold_merge(fa.R, fa.rows_R, fb.R, fb.rows_R, prec=prec)
    torch.cuda.synchronize()
    assert rows == 560
    X = torch.cat([xa, xb]).double()
    G = X.T @ X
    R = fa.R.double()
    assert float((R.T @ R - G).norm() / G.norm()) < tol
