"""Classic K-FAC comparator with the reference's API (``ifkfac/classic_kfac.py``,
``ifkfac/kfac_hooks.py``).

The control that IFKFAC is measured against: the Kronecker factors are formed
explicitly as Gram matrices A = X^T X / p and G = delta^T delta / p and
inverted, and the natural gradient is G^-1 grad A^-1.  Forming X^T X squares
the condition number, which in bf16 (the capture dtype under autocast) loses
the small eigen-directions; keeping that behaviour is the point of the
comparator, so the arithmetic is the reference's: a GEMM per chunk in the
capture dtype (``x.t().mm(x)``, ``kfac_hooks.py:211-219``) and an explicit
inverse of A + damping I (``classic_kfac.py:119-141``).

Differences that follow from running on the device:

* the Gram accumulation and the preconditioning are plain GEMMs (cuBLAS
  through torch); the inverse is taken in fp32 when the Gram matrix is bf16
  (``torch.linalg.inv`` has no bf16 kernel: the reference raises there), after
  the bf16 rounding of the Gram matrix that the comparison is about.
"""
from __future__ import annotations

import contextlib
import time
from collections import deque
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["KFACHooks", "ClassicKFAC"]


class KFACHooks:
    """Gram-matrix estimator (``ifkfac/kfac_hooks.py:67-297``): forward hooks
    accumulate A_sum += x^T x, full backward hooks G_sum += delta^T delta, per
    tracked nn.Linear / nn.Conv2d, with the row counts."""

    # 3-D (batch, seq, d) inputs: at most this many token rows per chunk (KFAC-Reduce,
    # kfac_hooks.py:176-188)
    _SEQ_SUBSAMPLE: int = 2048

    def __init__(self, model: nn.Module, max_gram_dim: int = 0):
        self.model = model
        self.max_gram_dim = max_gram_dim
        self._handles: List = []
        self._A_sum: Dict[nn.Module, torch.Tensor] = {}
        self._G_sum: Dict[nn.Module, torch.Tensor] = {}
        self._n_A: Dict[nn.Module, int] = {}
        self._n_G: Dict[nn.Module, int] = {}
        self._enabled = False
        self._linear_layers: List[nn.Module] = []
        for m in model.modules():
            if isinstance(m, (nn.Linear, nn.Conv2d)):
                out_dim = m.out_features if isinstance(m, nn.Linear) else m.out_channels
                if max_gram_dim > 0 and out_dim > max_gram_dim:
                    continue  # its G would be out_dim^2 (kfac_hooks.py:121-128)
                self._linear_layers.append(m)

    @property
    def linear_layers(self) -> List[nn.Module]:
        return self._linear_layers

    @property
    def is_enabled(self) -> bool:
        return self._enabled

    def enable(self) -> None:
        if self._enabled:
            return
        for m in self._linear_layers:
            self._handles.append(m.register_forward_hook(self._forward_hook))
            self._handles.append(m.register_full_backward_hook(self._backward_hook))
        self._enabled = True

    def pause(self) -> None:
        self._enabled = False

    def resume(self) -> None:
        self._enabled = True

    @contextlib.contextmanager
    def capture(self):
        """Capture for the duration of the block, then the previous state
        (``ifkfac/gram_estimator.py:150-175``)."""
        previous = self._enabled
        self._enabled = True
        try:
            yield self
        finally:
            self._enabled = previous

    @staticmethod
    def _rows_of_input(x: torch.Tensor, m: nn.Module) -> torch.Tensor:
        if isinstance(m, nn.Conv2d):  # im2col: (B * L, C_in * kH * kW) (kfac_hooks.py:151-167)
            u = F.unfold(x, kernel_size=m.kernel_size, dilation=m.dilation, padding=m.padding, stride=m.stride)
            return u.permute(0, 2, 1).reshape(-1, u.shape[1])
        return x.reshape(-1, x.shape[-1])

    @staticmethod
    def _rows_of_grad(d: torch.Tensor, m: nn.Module) -> torch.Tensor:
        if isinstance(m, nn.Conv2d):  # (B * H_out * W_out, C_out) (kfac_hooks.py:169-174)
            return d.permute(0, 2, 3, 1).reshape(-1, d.shape[1])
        return d.reshape(-1, d.shape[-1])

    def _subsample(self, rows: torch.Tensor, three_d: bool) -> torch.Tensor:
        if three_d and rows.shape[0] > self._SEQ_SUBSAMPLE:
            idx = torch.randperm(rows.shape[0], device=rows.device)[: self._SEQ_SUBSAMPLE]
            rows = rows[idx]
        return rows

    def _accumulate(self, sums, counts, m, rows):
        gram = rows.t().mm(rows)
        if m in sums:
            sums[m].add_(gram)
            counts[m] += rows.shape[0]
        else:
            sums[m] = gram
            counts[m] = rows.shape[0]

    def _forward_hook(self, m, inp, out):
        if not self._enabled:
            return
        x = inp[0].detach()
        rows = self._subsample(self._rows_of_input(x, m), not isinstance(m, nn.Conv2d) and x.ndim > 2)
        self._accumulate(self._A_sum, self._n_A, m, rows)

    def _backward_hook(self, m, grad_input, grad_output):
        if not self._enabled:
            return
        d = grad_output[0].detach()
        rows = self._subsample(self._rows_of_grad(d, m), not isinstance(m, nn.Conv2d) and d.ndim > 2)
        self._accumulate(self._G_sum, self._n_G, m, rows)

    def get_factors(self) -> Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]]:
        """(A_sum / n_A, G_sum / n_G) of every layer that saw a forward and a
        backward pass (``kfac_hooks.py:254-270``)."""
        return {m: (self._A_sum[m] / self._n_A[m], self._G_sum[m] / self._n_G[m])
                for m in self._linear_layers if m in self._A_sum and m in self._G_sum}

    def n_samples_accumulated(self, module: Optional[nn.Module] = None) -> int:
        target = module or (self._linear_layers[0] if self._linear_layers else None)
        return 0 if target is None else self._n_A.get(target, 0)

    def clear(self) -> None:
        self._A_sum.clear()
        self._G_sum.clear()
        self._n_A.clear()
        self._n_G.clear()

    def remove(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()
        self._enabled = False
        self.clear()


class ClassicKFAC(torch.optim.Optimizer):
    """K-FAC with explicit Gram inverses (``ifkfac/classic_kfac.py:25-306``):
    same constructor, schedule (factors when step % factor_update_freq == 1,
    inverses when step % decomp_update_freq == 1), EMA of the Gram matrices,
    decoupled weight decay, momentum on the weight only, bias preconditioned by
    G^-1, and plain SGD for layers without inverses yet."""

    def __init__(self, model: nn.Module, lr: float = 1e-3, damping: float = 1e-2, factor_update_freq: int = 10,
                 decomp_update_freq: int = 10, weight_decay: float = 0.0, momentum: float = 0.9,
                 grad_clip: Optional[float] = None, gamma: float = 0.0, max_gram_dim: int = 0):
        defaults = dict(lr=lr, damping=damping, weight_decay=weight_decay, momentum=momentum)
        params = [{"params": list(m.parameters())} for m in model.modules() if isinstance(m, (nn.Linear, nn.Conv2d))]
        super().__init__(params, defaults)
        self.model = model
        self.damping = damping
        self.factor_update_freq = factor_update_freq
        self.decomp_update_freq = decomp_update_freq
        self.grad_clip = grad_clip
        self.gamma = gamma
        self.hooks = KFACHooks(model, max_gram_dim=max_gram_dim)
        self.hooks.enable()
        self._factors: Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._inverses: Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._momentum_buffers: Dict[nn.Module, torch.Tensor] = {}
        self._step_count = 0
        self.timing = {k: deque(maxlen=1000) for k in ("factor_compute", "inversion", "precondition", "total_step")}

    def _group_of(self, p):
        for g in self.param_groups:
            if any(p is q for q in g["params"]):
                return g
        return None

    def _update_factors(self) -> None:
        """Gram factors of the window, EMA-blended with the previous ones when
        gamma > 0 (``classic_kfac.py:101-116``)."""
        t0 = time.perf_counter()
        new = self.hooks.get_factors()
        self.hooks.clear()
        if self.gamma > 0.0 and self._factors:
            for m, (A_new, G_new) in new.items():
                if m in self._factors:
                    A_old, G_old = self._factors[m]
                    new[m] = (self.gamma * A_old + (1.0 - self.gamma) * A_new,
                              self.gamma * G_old + (1.0 - self.gamma) * G_new)
        self._factors = new
        self.timing["factor_compute"].append(time.perf_counter() - t0)

    def _update_inverses(self) -> None:
        """inv(A + damping I), inv(G + damping I); non-finite factors are skipped
        (``classic_kfac.py:119-141``)."""
        t0 = time.perf_counter()
        for m, (A, G) in self._factors.items():
            if not (torch.isfinite(A).all() and torch.isfinite(G).all()):
                continue
            inv = []
            for M in (A, G):
                Md = M + self.damping * torch.eye(M.shape[0], device=M.device, dtype=M.dtype)
                inv.append(torch.linalg.inv(Md.float() if Md.dtype == torch.bfloat16 else Md))
            self._inverses[m] = (inv[0], inv[1])
        self.timing["inversion"].append(time.perf_counter() - t0)

    @torch.no_grad()
    def step(self, closure=None):
        t_total = time.perf_counter()
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._step_count += 1
        if self._step_count % self.factor_update_freq == 1 or self.factor_update_freq == 1:
            self._update_factors()
        if self._step_count % self.decomp_update_freq == 1 or self.decomp_update_freq == 1:
            if self._factors:
                self._update_inverses()
        t_pre = time.perf_counter()
        for m in self.hooks.linear_layers:
            if m not in self._inverses:
                for p in m.parameters():  # plain SGD with decoupled decay (classic_kfac.py:160-182)
                    g = self._group_of(p) if p.grad is not None else None
                    if g is None:
                        continue
                    if g["weight_decay"] > 0:
                        p.data.mul_(1.0 - g["lr"] * g["weight_decay"])
                    p.data.add_(p.grad, alpha=-g["lr"])
                continue
            A_inv, G_inv = self._inverses[m]
            g = self._group_of(m.weight)
            if g is None:
                continue
            lr, wd, mom = g["lr"], g["weight_decay"], g["momentum"]
            if m.weight.grad is not None:  # (classic_kfac.py:197-235)
                grad = m.weight.grad
                shape = grad.shape
                if grad.dim() > 2:
                    grad = grad.reshape(shape[0], -1)
                nat = (G_inv.to(grad.dtype) @ grad @ A_inv.to(grad.dtype)).reshape(shape)
                if self.grad_clip is not None:
                    norm = nat.norm()
                    if norm > self.grad_clip:
                        nat = nat * (self.grad_clip / norm)
                if mom > 0:
                    buf = self._momentum_buffers.get(m)
                    if buf is None:
                        buf = self._momentum_buffers[m] = torch.zeros_like(nat)
                    buf.mul_(mom).add_(nat)
                    nat = buf
                if wd > 0:
                    m.weight.data.mul_(1.0 - lr * wd)
                m.weight.data.add_(nat, alpha=-lr)
            if m.bias is not None and m.bias.grad is not None:  # no momentum on the bias (:237-243)
                nat_b = G_inv.to(m.bias.grad.dtype) @ m.bias.grad
                if wd > 0:
                    m.bias.data.mul_(1.0 - lr * wd)
                m.bias.data.add_(nat_b, alpha=-lr)
        self.timing["precondition"].append(time.perf_counter() - t_pre)
        self.timing["total_step"].append(time.perf_counter() - t_total)
        return loss

    def get_timing_stats(self) -> Dict[str, Dict[str, float]]:
        stats = {}
        for key, times in self.timing.items():
            if times:
                a = np.array(times)
                stats[key] = {"mean_ms": float(a.mean() * 1000), "p50_ms": float(np.percentile(a, 50) * 1000),
                              "p99_ms": float(np.percentile(a, 99) * 1000), "total_s": float(a.sum()),
                              "count": len(times)}
        return stats

    def capture(self):
        return self.hooks.capture()

    def pause_capture(self) -> None:
        self.hooks.pause()

    def resume_capture(self) -> None:
        self.hooks.resume()

    def cleanup(self) -> None:
        self.hooks.remove()
        self._factors.clear()
        self._inverses.clear()
        self._momentum_buffers.clear()

    def __repr__(self) -> str:
        return (f"ClassicKFAC(damping={self.damping}, factor_update_freq={self.factor_update_freq}, "
                f"decomp_update_freq={self.decomp_update_freq}, gamma={self.gamma}, "
                f"n_layers={len(self.hooks.linear_layers)})")
