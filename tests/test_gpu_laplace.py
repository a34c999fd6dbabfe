"""K-FAC Laplace posterior (ifkfac/laplace.py): the eigensolver-free draw
C_G^-1 xi C_A^-T from square roots of the factors (ifk_finalize + ifk_posterior_sample)
against the oracle, and the reference-API draw from eigendecompositions against
the reference's own golden draw."""
import math

import numpy as np
import pytest
import torch

from ifkfac_b200 import _lib
from ifkfac_b200.laplace import LaplacePosterior, posterior_factor, posterior_sample
from oracle import ifk_oracle as O
from tests.golden_io import load, rel

pytestmark = pytest.mark.gpu


def _R(n, seed):
    rng = np.random.default_rng(seed)
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    X = rng.standard_normal((3 * n, n)) * s
    return O.positive_diagonal_R(np.linalg.qr(X, mode="r")).astype(np.float32)


@pytest.mark.parametrize("dt,prec,tol", [(torch.float32, _lib.PREC_FP32, 1e-5), (torch.bfloat16, _lib.PREC_BF16, 2e-2)])
@pytest.mark.parametrize("n_out,n_in", [(96, 160), (300, 257), (1024, 512)])
def test_posterior_factor_and_draw_match_oracle(dt, prec, tol, n_out, n_in):
    N, lam = 5000, 0.3
    RA, RG = _R(n_in, 1 + n_in), _R(n_out, 2 + n_out)
    CA = posterior_factor(torch.from_numpy(RA).cuda(), N, lam, dt, prec)
    CG = posterior_factor(torch.from_numpy(RG).cuda(), N, lam, dt, prec)
    oA, oG = O.posterior_factor(RA.astype(np.float64), N, lam), O.posterior_factor(RG.astype(np.float64), N, lam)
    assert rel(CA.float().cpu().numpy(), oA) < tol
    assert rel(CG.float().cpu().numpy(), oG) < tol
    xi = torch.randn(n_out, n_in, generator=torch.Generator().manual_seed(3))
    dW = posterior_sample(xi.cuda(), CA, CG, prec)
    truth = O.posterior_sample(CA.double().cpu().numpy(), CG.double().cpu().numpy(), xi.double().numpy())
    assert rel(dW.cpu().numpy(), truth) < tol


def _golden_model(g):
    import torch.nn as nn
    model = nn.Sequential(nn.Linear(12, 16), nn.ReLU(), nn.Linear(16, 6)).cuda()
    layers = [model[0], model[2]]
    with torch.no_grad():
        for i, m in enumerate(layers):
            m.weight.copy_(torch.from_numpy(g[f"Wmap{i}"]))
    return model, layers


def test_evd_draw_matches_reference_golden():
    """The reference constructor: its draw for the recorded xi gives the reference's weights."""
    g = load("laplace")
    N, lam = int(g["N"]), float(g["lam"])
    model, layers = _golden_model(g)
    evd = {m: tuple(torch.from_numpy(g[f"{k}{i}"]).cuda() for k in ("U_A", "d_A", "U_G", "d_G"))
           for i, m in enumerate(layers)}
    post = LaplacePosterior(model, evd, prior_precision=lam, dataset_size=N)
    for i, m in enumerate(layers):
        dW = post.perturbation(m, torch.from_numpy(g[f"xi{i}"]).cuda())
        assert rel(g[f"Wmap{i}"] + dW.cpu().numpy(), g[f"Wsample{i}"]) < 1e-5


@pytest.mark.parametrize("precision", [_lib.PREC_FP32, _lib.PREC_BF16])
def test_from_R_posterior_lifecycle(precision):
    """from_R on the golden layers: the per-side precision is the reference's
    U diag(sqrt(N) d + sqrt(lambda)) U^T; draws change the weights, restore_map
    brings the MAP back, predictive is a distribution."""
    g = load("laplace")
    N, lam = int(g["N"]), float(g["lam"])
    model, layers = _golden_model(g)
    facs = {m: (torch.from_numpy(g[f"R_A{i}"]).cuda(), torch.from_numpy(g[f"R_G{i}"]).cuda())
            for i, m in enumerate(layers)}
    post = LaplacePosterior.from_R(model, facs, prior_precision=lam, dataset_size=N, precision=precision)
    tol = 1e-5 if precision == _lib.PREC_FP32 else 2e-2
    for i, m in enumerate(layers):
        CA, CG = (c.double().cpu().numpy() for c in post._tri[m])
        for C, tag in ((CA, "A"), (CG, "G")):
            U, d = g[f"U_{tag}{i}"].astype(np.float64), g[f"d_{tag}{i}"].astype(np.float64)
            P = U @ np.diag(math.sqrt(N) * d + math.sqrt(lam)) @ U.T
            assert rel(C.T @ C, P) < 2 * tol
        xi = torch.from_numpy(g[f"xi{i}"]).cuda()
        dW = post.perturbation(m, xi).cpu().numpy()
        assert rel(dW, O.posterior_sample(CA, CG, g[f"xi{i}"].astype(np.float64))) < tol
    w0 = [m.weight.detach().clone() for m in layers]
    post.sample_in_place(generator=torch.Generator(device="cuda").manual_seed(1))
    assert all(not torch.equal(m.weight, w) for m, w in zip(layers, w0))
    post.restore_map()
    assert all(torch.equal(m.weight, w) for m, w in zip(layers, w0))
    x = torch.randn(32, 12, device="cuda")
    p = post.predictive(x, n_samples=4, generator=torch.Generator(device="cuda").manual_seed(2))
    assert p.shape == (32, 6)
    assert torch.allclose(p.sum(-1), torch.ones(32, device="cuda"), atol=1e-5)
    assert all(torch.equal(m.weight, w) for m, w in zip(layers, w0))


def test_draw_covariance_matches_posterior():
    """Monte-Carlo check of the distribution: the sample covariance of many
    draws of a small layer matches P_A^-1 (x) P_G^-1 (columns and rows)."""
    N, lam, n_out, n_in = 40, 0.7, 6, 5
    RA, RG = _R(n_in, 7), _R(n_out, 8)
    CA = posterior_factor(torch.from_numpy(RA).cuda(), N, lam)
    CG = posterior_factor(torch.from_numpy(RG).cuda(), N, lam)
    S = 2000
    xi = torch.randn(S * n_out, n_in, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    d = torch.stack([posterior_sample(xi[s * n_out:(s + 1) * n_out], CA, CG) for s in range(S)])
    flat = d.reshape(d.shape[0], -1).double().cpu().numpy()
    cov = flat.T @ flat / flat.shape[0]
    PA = O.posterior_factor(RA.astype(np.float64), N, lam)
    PG = O.posterior_factor(RG.astype(np.float64), N, lam)
    SA, SG = np.linalg.inv(PA.T @ PA), np.linalg.inv(PG.T @ PG)
    truth = np.kron(SG, SA)  # vec over rows of W (row-major): Cov[W_ij, W_kl] = SG_ik SA_jl
    assert rel(cov, truth) < 0.1


@pytest.mark.parametrize("dt,prec", [(torch.float32, _lib.PREC_FP32), (torch.bfloat16, _lib.PREC_BF16)])
def test_batched_factors_equal_single(dt, prec):
    """posterior_factors (one ifk_finalize_many call) gives each factor of posterior_factor."""
    from ifkfac_b200.laplace import posterior_factors
    Rs = [torch.from_numpy(_R(n, 30 + n)).cuda() for n in (64, 200, 96, 513)]
    st = torch.zeros(len(Rs), dtype=torch.int32, device="cuda")
    many = posterior_factors(Rs, 1000, 0.1, dt, prec, st)
    torch.cuda.synchronize()
    assert st.tolist() == [0] * len(Rs)
    for R, C in zip(Rs, many):
        one = posterior_factor(R, 1000, 0.1, dt, prec)
        assert float((C.float() - one.float()).norm() / one.float().norm()) < 1e-6
