"""Classic K-FAC comparator on the GPU, and the contrast it exists for
(the reference's tests/test_bf16_stability.py, whose bf16 case does not run
there): at bf16 and kappa = 100, forming the Gram matrix squares the condition
number and its inverse loses the preconditioner, while the QR route of the
bf16 tensor-core kernels keeps it."""
import math

import pytest
import torch

from ifkfac_b200 import _lib
from ifkfac_b200.engine import Factor, fold_segments
from ifkfac_b200.triangular import apply_vered, damped_factor
from tests.test_classic import run_classic

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tag", ["mlp", "conv"])
def test_classic_trajectory_matches_reference_gpu(tag):
    errs, _ = run_classic(tag, "cuda")
    assert max(e for _, _, e in errs) < 1e-4, max(errs, key=lambda t: t[2])


def _with_kappa(p, n, kappa, seed):
    g = torch.Generator().manual_seed(seed)
    U, _ = torch.linalg.qr(torch.randn(p, n, generator=g, dtype=torch.float64))
    V, _ = torch.linalg.qr(torch.randn(n, n, generator=g, dtype=torch.float64))
    return U @ torch.diag(torch.logspace(0, math.log10(kappa), n, dtype=torch.float64)) @ V.T


@pytest.mark.parametrize("kappa", [10.0, 100.0])
def test_bf16_stability_contrast(kappa):
    p, n_in, n_out, lam = 4096, 256, 192, 1e-3
    X, D = _with_kappa(p, n_in, kappa, 1), _with_kappa(p, n_out, kappa, 2)
    grad = torch.randn(n_out, n_in, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    Xb, Db = X.to(torch.bfloat16), D.to(torch.bfloat16)  # the captured bf16 rows both methods see
    Xe, De = Xb.double(), Db.double()
    A = Xe.T @ Xe / p + lam * torch.eye(n_in, dtype=torch.float64)
    G = De.T @ De / p + lam * torch.eye(n_out, dtype=torch.float64)
    truth = torch.linalg.solve(G, grad) @ torch.linalg.inv(A)
    # Classic in bf16: the Gram matrices formed from the bf16 rows on the device, kept in bf16
    # (kfac_hooks.py:211-219 under autocast), inverted (ClassicKFAC._update_inverses)
    Xc, Dc = Xb.cuda(), Db.cuda()
    Ab = (Xc.t().mm(Xc) / p) + lam * torch.eye(n_in, device="cuda", dtype=torch.bfloat16)
    Gb = (Dc.t().mm(Dc) / p) + lam * torch.eye(n_out, device="cuda", dtype=torch.bfloat16)
    classic = torch.linalg.inv(Gb.float()) @ grad.float().cuda() @ torch.linalg.inv(Ab.float())
    # IFKFAC in bf16 mode: the rows folded on the tensor cores, bf16 damped factors, bf16-mode solves
    facs = []
    for rows, n in ((Xc, n_in), (Dc, n_out)):
        f = Factor(n, "cuda", _lib.PREC_BF16)
        fold_segments((f,), ([rows],), None)
        facs.append(damped_factor(f.R, f.rows_R, p, lam, torch.bfloat16, _lib.PREC_BF16))
    ours = apply_vered(grad.float().cuda(), facs[0], facs[1], prec=_lib.PREC_BF16)
    err = lambda a: float((a.double().cpu() - truth).norm() / truth.norm())
    e_classic, e_ours = err(classic), err(ours)
    print(f"kappa {kappa}: classic bf16 {e_classic:.3e}, ifkfac bf16 {e_ours:.3e}")
    assert e_ours < 2e-2, e_ours
    if kappa >= 100:
        assert e_classic > 5 * e_ours, (e_classic, e_ours)
