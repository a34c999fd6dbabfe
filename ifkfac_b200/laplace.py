"""K-FAC Laplace posterior with the reference's API (``ifkfac/laplace.py``).

The posterior over a layer's weights is N(W_map, Sigma) with the Kronecker
covariance Sigma = P_A^-1 (x) P_G^-1 of the per-side precisions

    P_A = sqrt(N) A + sqrt(lambda) I,   P_G = sqrt(N) G + sqrt(lambda) I

(Daxberger et al. 2021, section 4 and appendix A; ``ifkfac/laplace.py:1-37``).
The reference takes eigendecompositions A = U_A diag(d_A) U_A^T (and G) and
draws W_map + U_G diag(s_G) Xi diag(s_A) U_A^T with s = (sqrt(N) d + sqrt(lambda))^-1/2
(``:96-109``, ``:127-146``).  Its IFKFAC variant gets the eigendecomposition
from svd(R) of the factor's square root R (R^T R = A, ``:27-29``).

Two ways in:

* ``LaplacePosterior(model, factors_evd, ...)``: the reference's constructor and
  draw, from eigendecompositions; the draw is two GEMMs per layer.
* ``LaplacePosterior.from_R(model, factors_R, ...)``: from the square roots
  themselves (R_A^T R_A = A, as the hooks hold them), with no eigensolver.
  P_A = C_A^T C_A for the upper-triangular C_A = qr([N^1/4 R_A; lambda^1/4 I]),
  which is the damping fold of ``ifk_finalize`` (rows_total N^-1/2, damping
  sqrt(lambda)); a draw is W_map + C_G^-1 Xi C_A^-T, two blocked triangular
  solves (``ifk_posterior_sample``).  Its covariance is the same P_A^-1 (x) P_G^-1:
  the same posterior from another square root, so individual draws for a given
  Xi differ from the eigenbasis form while their distribution does not.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn

from . import _lib
from ._lib import check
from .triangular import _code, _need_cuda, _rows_contig, _stream, _workspace, damped_factor

__all__ = ["LaplacePosterior", "posterior_factor", "posterior_factors", "posterior_sample"]

EVDFactor = Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]


def posterior_factor(R: torch.Tensor, dataset_size: int, prior_precision: float,
                     out_dtype: torch.dtype = torch.float32, prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """Upper-triangular C (positive diagonal) with C^T C = sqrt(N) R^T R + sqrt(lambda) I,
    the posterior precision of one side for A = R^T R (``ifkfac/laplace.py:96-109``):
    ``ifk_finalize`` of R with rows_total N^-1/2 and damping sqrt(lambda)."""
    _need_cuda(R)
    n = R.shape[0]
    if R.dim() != 2 or R.shape[1] != n:
        raise ValueError(f"R must be square, got {tuple(R.shape)}")
    Rf = R.float().contiguous()
    out = damped_factor(Rf, n, float(dataset_size) ** -0.5, float(prior_precision) ** 0.5, out_dtype, prec)
    assert out is not None
    return out


def posterior_factors(Rs, dataset_size: int, prior_precision: float, out_dtype: torch.dtype = torch.float32,
                      prec: int = _lib.PREC_AUTO, status: Optional[torch.Tensor] = None):
    """posterior_factor of every R in Rs by one ``ifk_finalize_many`` call (the damping
    folds of up to 16 factors share a launch).  ``status`` (int32, one word per R,
    zeroed here when given) receives each factor's non-finite / timeout code."""
    Rs = [R.float().contiguous() for R in Rs]
    if not Rs:
        return []
    _need_cuda(*Rs)
    for R in Rs:
        if R.dim() != 2 or R.shape[0] != R.shape[1]:
            raise ValueError(f"R must be square, got {tuple(R.shape)}")
    dev = Rs[0].device
    if status is None:
        status = torch.zeros(len(Rs), dtype=torch.int32, device=dev)
    else:
        status.zero_()
    arr = lambda t, v: (t * len(v))(*v)
    ns = [R.shape[0] for R in Rs]
    outs = [torch.empty(n, n, dtype=out_dtype, device=dev) for n in ns]
    L = _lib.lib()
    ws = _workspace(L.ifk_finalize_batched_workspace(len(Rs), arr(ctypes.c_int64, ns)), dev)
    check(L.ifk_finalize_many(
        len(Rs), arr(ctypes.c_void_p, [R.data_ptr() for R in Rs]), arr(ctypes.c_int64, [R.stride(0) for R in Rs]),
        arr(ctypes.c_int64, ns), arr(ctypes.c_int64, ns), arr(ctypes.c_double, [float(dataset_size) ** -0.5] * len(Rs)),
        float(prior_precision) ** 0.5, arr(ctypes.c_void_p, [o.data_ptr() for o in outs]), arr(ctypes.c_int64, ns),
        _code(outs[0]), prec, arr(ctypes.c_void_p, [status.data_ptr() + 4 * i for i in range(len(Rs))]),
        ws.data_ptr(), ws.numel(), _stream()), "ifk_finalize_many")
    return outs


def posterior_sample(xi: torch.Tensor, C_A: torch.Tensor, C_G: torch.Tensor,
                     prec: int = _lib.PREC_AUTO, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C_G^-1 xi C_A^-T (n_out x n_in fp32): a draw of covariance
    (C_A^T C_A)^-1 (x) (C_G^T C_G)^-1 when xi is iid N(0, 1)."""
    _need_cuda(xi, C_A, C_G)
    n_out, n_in = xi.shape
    if C_A.shape != (n_in, n_in) or C_G.shape != (n_out, n_out) or C_A.dtype != C_G.dtype:
        raise ValueError("C_A (n_in x n_in) and C_G (n_out x n_out) of one dtype")
    out = xi.float().contiguous().clone()
    C_A, C_G = _rows_contig(C_A), _rows_contig(C_G)
    L = _lib.lib()
    ws = _workspace(L.ifk_posterior_sample_workspace(n_out, n_in), xi.device)
    sp = status.data_ptr() if status is not None else None
    check(L.ifk_posterior_sample(out.data_ptr(), out.stride(0), C_A.data_ptr(), C_A.stride(0),
                                 C_G.data_ptr(), C_G.stride(0), _code(C_A), out.data_ptr(), out.stride(0),
                                 n_out, n_in, prec, sp, ws.data_ptr(), ws.numel(), _stream()),
          "ifk_posterior_sample")
    return out


class LaplacePosterior:
    """K-FAC Laplace posterior (``ifkfac/laplace.py:58-226``).

    Parameters as the reference's: ``factors_evd`` maps a layer to
    (U_A, d_A, U_G, d_G); ``prior_precision`` is lambda; ``dataset_size`` is N
    (eigenvalues scaled by sqrt(N), ``:70-79``).  See :meth:`from_R` for the
    eigensolver-free form."""

    def __init__(self, model: nn.Module, factors_evd: Dict[nn.Module, EVDFactor],
                 prior_precision: float = 1.0, dataset_size: int = 1):
        self.model = model
        self.prior_precision = prior_precision
        self.dataset_size = dataset_size
        self._w_map: Dict[nn.Module, torch.Tensor] = {m: m.weight.data.clone() for m in factors_evd}
        sqrt_N, sqrt_lam = float(dataset_size) ** 0.5, float(prior_precision) ** 0.5
        # (U_A, s_A, U_G, s_G) with s = 1 / sqrt(sqrt(N) d + sqrt(lambda)) (:96-109)
        self._evd: Dict[nn.Module, EVDFactor] = {}
        for m, (U_A, d_A, U_G, d_G) in factors_evd.items():
            self._evd[m] = (U_A.float(), (1.0 / torch.sqrt(sqrt_N * d_A + sqrt_lam)).float(),
                            U_G.float(), (1.0 / torch.sqrt(sqrt_N * d_G + sqrt_lam)).float())
        self._tri: Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._prec = _lib.PREC_AUTO

    @classmethod
    def from_R(cls, model: nn.Module, factors_R: Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]],
               prior_precision: float = 1.0, dataset_size: int = 1,
               precision: int = _lib.PREC_AUTO) -> "LaplacePosterior":
        """The posterior from square roots R_A, R_G of each layer's factors
        (R_A^T R_A = A: the hooks' factors at damping 0, or their running R
        scaled by 1/sqrt(rows)).  ``precision``: ``_lib.PREC_BF16`` keeps C_A, C_G
        in bf16 and solves on the tensor cores (bf16 R selects it too);
        ``_lib.PREC_FP32`` keeps them fp32.  All factors are built by one
        ``ifk_finalize_many`` call; ``self.status`` holds a status word per factor
        (layer i: 2i for C_A, 2i + 1 for C_G; non-zero: not finite / timed out)."""
        self = cls(model, {}, prior_precision, dataset_size)
        mods = list(factors_R)
        if not mods:
            return self
        R0 = factors_R[mods[0]][0]
        bf16 = precision == _lib.PREC_BF16 or (precision == _lib.PREC_AUTO and R0.dtype == torch.bfloat16)
        dt = torch.bfloat16 if bf16 else torch.float32
        self._prec = _lib.PREC_BF16 if bf16 else _lib.PREC_FP32
        # every layer's two factors in one call; status word 2i / 2i + 1 for layer i
        self.status = torch.zeros(2 * len(mods), dtype=torch.int32, device=R0.device)
        Cs = posterior_factors([R for m in mods for R in factors_R[m]], dataset_size, prior_precision, dt,
                               self._prec, self.status)
        for i, m in enumerate(mods):
            self._tri[m] = (Cs[2 * i], Cs[2 * i + 1])
            self._w_map[m] = m.weight.data.clone()
        return self

    def _layers(self):
        return list(self._evd) + [m for m in self._tri if m not in self._evd]

    @torch.no_grad()
    def perturbation(self, module: nn.Module, xi: torch.Tensor) -> torch.Tensor:
        """The weight perturbation of one layer for the standard-normal matrix xi
        (n_out x n_in): U_G diag(s_G) xi diag(s_A) U_A^T (``:136-146``), or
        C_G^-1 xi C_A^-T for a posterior built by :meth:`from_R`."""
        if module in self._tri:
            C_A, C_G = self._tri[module]
            pr = _lib.PREC_BF16 if C_A.dtype == torch.bfloat16 else _lib.PREC_FP32
            return posterior_sample(xi, C_A, C_G, pr)
        U_A, s_A, U_G, s_G = self._evd[module]
        xs = xi.float() * s_G.unsqueeze(1) * s_A.unsqueeze(0)
        return U_G @ xs @ U_A.t()

    @torch.no_grad()
    def sample_in_place(self, generator: Optional[torch.Generator] = None) -> None:
        """Draw one weight sample per layer into the model (``:112-159``): restore
        W_map, draw xi ~ N(0, I) of shape (n_out, n_in), add the perturbation.
        Layers without factors keep their MAP values."""
        for m in self._layers():
            W = m.weight
            n_out = W.shape[0]
            n_in = W[0].numel()
            W.data.copy_(self._w_map[m])
            xi = torch.randn(n_out, n_in, device=W.device, dtype=torch.float32, generator=generator)
            dW = self.perturbation(m, xi)
            if W.ndim > 2:  # Conv2d: (C_out, C_in*kH*kW) -> the weight's shape (:147-149)
                dW = dW.reshape(W.data.shape)
            W.data.add_(dW.to(W.dtype))

    @torch.no_grad()
    def restore_map(self) -> None:
        """Reset weights to the MAP point (``:161-165``)."""
        for m in self._layers():
            m.weight.data.copy_(self._w_map[m])

    @torch.no_grad()
    def predictive(self, x: torch.Tensor, n_samples: int = 30,
                   generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """Single-batch Monte-Carlo predictive (``:167-190``): mean softmax over
        n_samples weight draws, then the MAP weights back."""
        was_training = self.model.training
        self.model.eval()
        probs_sum = None
        for _ in range(n_samples):
            self.sample_in_place(generator=generator)
            p = torch.softmax(self.model(x).float(), dim=-1)
            probs_sum = p if probs_sum is None else probs_sum + p
        self.restore_map()
        if was_training:
            self.model.train()
        return probs_sum / n_samples

    @torch.no_grad()
    def predictive_full_loader(self, loader, device, n_samples: int = 30,
                               generator: Optional[torch.Generator] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Monte-Carlo predictive over a whole loader with n_samples weight draws in
        total (``:192-226``); returns (probs (N_total, n_classes), labels)."""
        was_training = self.model.training
        self.model.eval()
        probs_sum, labels_all = None, None
        for _ in range(n_samples):
            self.sample_in_place(generator=generator)
            batch_probs, batch_labels = [], ([] if labels_all is None else None)
            for x, y in loader:
                logits = self.model(x.to(device, non_blocking=True))
                batch_probs.append(torch.softmax(logits.float(), dim=-1).cpu())
                if batch_labels is not None:
                    batch_labels.append(y)
            all_probs = torch.cat(batch_probs)
            probs_sum = all_probs if probs_sum is None else probs_sum + all_probs
            if labels_all is None:
                labels_all = torch.cat(batch_labels)
        self.restore_map()
        if was_training:
            self.model.train()
        return probs_sum / n_samples, labels_all
