"""IFKFAC optimizer on the B200 curvature library.

Mirror of the reference's ``IFKFAC`` (ifkfac/ifkfac.py:78-642): the same
constructor ``IFKFAC(model, lr, damping, factor_update_freq, weight_decay,
momentum, grad_clip, gamma, max_out_dim, augment_bias, max_conv_rows,
max_seq_rows, batched_qr, deferred_qr, use_true_bf16)``, the same step()
schedule (factor refresh every step when factor_update_freq == 1, else at
step >= freq with step % freq == 0; plain SGD without momentum before the
first refresh), the same per-layer epilogue (natural-gradient norm clip,
momentum, decoupled weight decay, lr step, bias through R_G only) and the
same fallbacks (rank-deficient layers keep accumulating, non-finite factors
are skipped, a failed solve uses the raw gradient).  The linear algebra runs
in libifk.so on CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import ctypes
import logging
import math
import time
import warnings
from collections import deque
from typing import Dict, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from . import _lib
from ._lib import IFKError, check
from .activation_hooks import IFKFACRankError, RawActivationHooks
from .engine import Factor, fold_batched

logger = logging.getLogger(__name__)

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def should_refresh(step_count: int, factor_update_freq: int) -> bool:
    """ifkfac/ifkfac.py:560-564."""
    if factor_update_freq == 1:
        return True
    return step_count >= factor_update_freq and step_count % factor_update_freq == 0


class IFKFAC(torch.optim.Optimizer):
    """K-FAC with QR factors and triangular solves (no explicit inverse), on B200."""

    def __init__(self, model: nn.Module, lr: float = 1e-3, damping: float = 1e-2,
                 factor_update_freq: int = 10, weight_decay: float = 0.0, momentum: float = 0.9,
                 grad_clip: Optional[float] = None, gamma: float = 0.0, max_out_dim: int = 0,
                 augment_bias: bool = False, max_conv_rows: int = 512,
                 max_seq_rows: Optional[int] = None, batched_qr: bool = False,
                 deferred_qr: bool = False, use_true_bf16: bool = False,
                 precision: int = _lib.PREC_AUTO):
        self.use_true_bf16 = use_true_bf16
        params = []
        for module in model.modules():
            if isinstance(module, (nn.Linear, nn.Conv2d)):
                params.append({"params": list(module.parameters())})
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, momentum=momentum))
        self.model = model
        self.damping = damping
        self.factor_update_freq = factor_update_freq
        self.grad_clip = grad_clip
        self.gamma = gamma
        self.augment_bias = augment_bias
        # use_true_bf16 asks for bf16 factors: their folds run in bf16 mode (tensor cores)
        # whatever the dtype of the captured rows, unless a precision is given
        if use_true_bf16 and precision == _lib.PREC_AUTO:
            precision = _lib.PREC_BF16
        self.precision = precision
        self.hooks = RawActivationHooks(model, damping=damping, max_out_dim=max_out_dim,
                                        augment_bias=augment_bias, max_conv_rows=max_conv_rows,
                                        max_seq_rows=max_seq_rows, batched=batched_qr,
                                        deferred=deferred_qr, precision=precision)
        self.hooks.enable()
        self._factors: Dict[nn.Module, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._classic_fallback: Dict = {}
        self._momentum_buffers: Dict[nn.Module, torch.Tensor] = {}
        self._ws: Dict = {}
        self._step_count = 0
        self.timing = {k: deque(maxlen=1000) for k in ("factor_compute", "precondition", "total_step")}

    # ---- factor refresh (ifkfac/ifkfac.py:202-302) ----
    def _update_factors(self) -> None:
        t0 = time.perf_counter()
        try:
            new = self.hooks.get_factors()
        except IFKFACRankError as e:
            logger.warning("IFKFAC: factor update skipped — %s", e)
            self.timing["factor_compute"].append(time.perf_counter() - t0)
            return
        self.hooks.clear()
        clean = {}
        if new:
            st = self.hooks.last_status.cpu().numpy()   # one sync, like isfinite().all()
            for module, pair in new.items():
                if st[self.hooks.status_index[module]] != 0:
                    logger.warning("IFKFAC: non-finite R for layer %s — skipping.", type(module).__name__)
                    continue
                clean[module] = pair
        if self.gamma > 0.0 and self._factors:
            clean = {m: (self._blend(self._factors[m][0], rx), self._blend(self._factors[m][1], rg))
                     if m in self._factors else (rx, rg) for m, (rx, rg) in clean.items()}
        if self.use_true_bf16:
            clean = {m: (rx.to(torch.bfloat16), rg.to(torch.bfloat16)) for m, (rx, rg) in clean.items()}
        self._factors = clean
        self.timing["factor_compute"].append(time.perf_counter() - t0)

    def _blend(self, R_old: torch.Tensor, R_new: torch.Tensor) -> torch.Tensor:
        """Exact EMA blend (ifkfac/ifkfac.py:261-285): R of [sqrt(g) R_old; sqrt(1-g) R_new],
        a fold of the scaled new factor (trapezoidal chunk) into the scaled old one."""
        n = R_new.shape[0]
        f = Factor(n, R_new.device, self.precision)
        f.R.copy_(R_old.float() * math.sqrt(self.gamma))
        f.rows_R = n
        fold_batched([f], [(R_new.float() * math.sqrt(1.0 - self.gamma)).contiguous()], None,
                     trapezoidal=True)
        return f.R

    # ---- preconditioner apply (ifkfac/ifkfac.py:315-519) ----
    def _get_module_hp(self, module):
        for group in self.param_groups:
            if any(p is module.weight for p in group["params"]):
                return group["lr"], group["weight_decay"], group["momentum"]
        return None, None, None

    def _workspace(self, key, nbytes, device):
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def _natgrad(self, g: torch.Tensor, R_X: torch.Tensor, R_G: torch.Tensor) -> torch.Tensor:
        L = _lib.lib()
        n_out, n_in = g.shape
        if R_X.dtype != R_G.dtype:
            R_X, R_G = R_X.float(), R_G.float()
        R_X, R_G = R_X.contiguous(), R_G.contiguous()
        g32 = g.float().contiguous()
        nat = torch.empty_like(g32)
        ws = self._workspace(("nat", g.device), L.ifk_natgrad_workspace(n_out, n_in), g.device)
        check(L.ifk_natgrad(g32.data_ptr(), n_in, R_X.data_ptr(), n_in, R_G.data_ptr(), n_out,
                            _DT[R_X.dtype], nat.data_ptr(), n_in, n_out, n_in, self.precision, None,
                            ws.data_ptr(), ws.numel(), _stream()), "ifk_natgrad")
        return nat

    def _natgrad_many(self, items, biases=None):
        """Natural gradients of several layers with one ifk_natgrad_batched call:
        items are (g, R_X, R_G) with factors of one dtype on one device; biases
        (optional, an entry per layer, None where a layer has no bias gradient)
        come back solved by R_G^-1 R_G^-T as the second list."""
        import ctypes
        L = _lib.lib()
        arr = lambda t, v: (t * len(v))(*v)
        gs = [g.float().contiguous() for g, _, _ in items]
        rx = [R_X.contiguous() for _, R_X, _ in items]
        rg = [R_G.contiguous() for _, _, R_G in items]
        nats = [torch.empty_like(g) for g in gs]
        bs = [b.float().contiguous() if b is not None else None for b in (biases or [None] * len(gs))]
        nbs = [torch.empty_like(b) if b is not None else None for b in bs]
        ptr = lambda t: t.data_ptr() if t is not None else None
        n_out = [g.shape[0] for g in gs]
        n_in = [g.shape[1] for g in gs]
        dev = gs[0].device
        ws = self._workspace(("natb", dev), L.ifk_natgrad_batched_workspace(
            len(gs), arr(ctypes.c_int64, n_out), arr(ctypes.c_int64, n_in)), dev)
        check(L.ifk_natgrad_batched(
            len(gs), arr(ctypes.c_void_p, [g.data_ptr() for g in gs]), arr(ctypes.c_int64, n_in),
            arr(ctypes.c_void_p, [r.data_ptr() for r in rx]), arr(ctypes.c_int64, n_in),
            arr(ctypes.c_void_p, [r.data_ptr() for r in rg]), arr(ctypes.c_int64, n_out), _DT[rx[0].dtype],
            arr(ctypes.c_void_p, [o.data_ptr() for o in nats]), arr(ctypes.c_int64, n_in),
            arr(ctypes.c_int64, n_out), arr(ctypes.c_int64, n_in), arr(ctypes.c_void_p, [ptr(b) for b in bs]),
            arr(ctypes.c_void_p, [ptr(b) for b in nbs]), self.precision, None, ws.data_ptr(),
            ws.numel(), _stream()), "ifk_natgrad_batched")
        return nats, nbs

    def _natgrad_bias(self, gb: torch.Tensor, R_G: torch.Tensor) -> torch.Tensor:
        L = _lib.lib()
        R_G = R_G.contiguous()
        g32 = gb.float().contiguous()
        out = torch.empty_like(g32)
        check(L.ifk_natgrad_bias(g32.data_ptr(), R_G.data_ptr(), R_G.shape[0], _DT[R_G.dtype],
                                 out.data_ptr(), R_G.shape[0], self.precision, None, 0, _stream()),
              "ifk_natgrad_bias")
        return out

    def _update_param(self, p: torch.Tensor, step: torch.Tensor, lr, wd, mom, buf_owner=None,
                      clip: Optional[float] = None) -> None:
        """ifk_update on fp32 master weights; momentum only when buf_owner is given."""
        L = _lib.lib()
        data = p.data
        if data.dtype != torch.float32 or not data.is_contiguous():
            # non-fp32 or strided parameters: same arithmetic with torch ops on the device
            g = step.to(data.dtype)
            if clip is not None:
                gn = g.float().norm()
                if gn > clip:
                    g = g * (clip / gn)
            if mom > 0 and buf_owner is not None:
                buf = self._momentum_buffers.get(buf_owner)
                if buf is None:
                    buf = self._momentum_buffers[buf_owner] = torch.zeros_like(g)
                buf.mul_(mom).add_(g)
                g = buf
            if wd > 0:
                data.mul_(1.0 - lr * wd)
            data.add_(g, alpha=-lr)
            return
        step = step.float().contiguous().view(-1)
        use_mom = mom > 0 and buf_owner is not None
        new = False
        buf = None
        if use_mom:
            buf = self._momentum_buffers.get(buf_owner)
            if buf is None:
                buf = self._momentum_buffers[buf_owner] = torch.empty_like(data)
                new = True
        ws = self._workspace(("upd", data.device), 256, data.device) if clip else None
        check(L.ifk_update(data.data_ptr(), buf.data_ptr() if use_mom else None, step.data_ptr(),
                           data.numel(), float(lr), float(mom) if use_mom else 0.0, float(wd),
                           float(clip) if clip else 0.0, 1 if new else 0,
                           ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                           _stream()), "ifk_update")

    def _layer_factors(self, module):
        """(g2, R_X, R_G) of a layer that has square factors, else None."""
        if module not in self._factors or module.weight.grad is None:
            return None
        R_X, R_G = self._factors[module]
        if self.augment_bias and module.bias is not None:
            R_X = R_X[:-1, :-1].contiguous()
        if R_X.shape[0] != R_X.shape[1] or R_G.shape[0] != R_G.shape[1] or R_X.dtype != R_G.dtype:
            return None
        grad_w = module.weight.grad
        g2 = grad_w.reshape(grad_w.shape[0], -1) if grad_w.dim() > 2 else grad_w
        return g2, R_X, R_G

    def _batched_natgrads(self, modules) -> dict:
        """Natural gradients of every layer with square factors, the layers of one
        factor dtype and device in one batched call (the bucketed apply of
        ifkfac/ifkfac.py:315-423); a failed batch leaves its layers to the
        per-layer path."""
        groups = {}
        for m in modules:
            it = self._layer_factors(m)
            if it is not None:
                groups.setdefault((it[1].dtype, it[1].device), []).append((m, it))
        out = {}
        for lst in groups.values():
            if len(lst) < 2:
                continue
            biases = [m.bias.grad if m.bias is not None and m.bias.grad is not None else None for m, _ in lst]
            try:
                nats, nbs = self._natgrad_many([it for _, it in lst], biases)
            except IFKError as e:
                logger.warning("IFKFAC: batched apply_vered failed (%s) — layers go one by one.", e)
                continue
            for (m, _), nat, nb in zip(lst, nats, nbs):
                out[m] = (nat, nb)
        return out

    def _apply_preconditioner(self, module, lr, weight_decay, momentum, pre=None) -> None:
        """pre: (natural gradient of the weight, of the bias or None) from the batched apply."""
        nat_pre, nb_pre = pre if pre is not None else (None, None)
        weight = module.weight
        if weight.grad is None:
            return
        if module not in self._factors:
            # no preconditioner yet: plain SGD on the weight only, no momentum, decoupled
            # decay; the bias is left as is (ifkfac/ifkfac.py:443-448)
            self._update_param(weight, weight.grad, lr, weight_decay, 0.0)
            return
        R_X, R_G = self._factors[module]
        if self.augment_bias and module.bias is not None:
            R_X = R_X[:-1, :-1].contiguous()
        grad_w = weight.grad
        g2 = grad_w.reshape(grad_w.shape[0], -1) if grad_w.dim() > 2 else grad_w
        try:
            if nat_pre is not None:
                nat = nat_pre
            elif R_X.shape[0] != R_X.shape[1] or R_G.shape[0] != R_G.shape[1]:
                nat = g2.float()
            else:
                nat = self._natgrad(g2, R_X, R_G)
        except IFKError as e:
            logger.warning("IFKFAC: apply_vered failed for %s (%s) — using raw gradient.",
                           type(module).__name__, e)
            nat = g2.float()
        self._update_param(weight, nat.reshape(grad_w.shape), lr, weight_decay, momentum,
                           buf_owner=module, clip=self.grad_clip)
        if module.bias is not None and module.bias.grad is not None:
            try:
                nb = nb_pre if nb_pre is not None else self._natgrad_bias(module.bias.grad, R_G)
            except IFKError as e:
                logger.warning("IFKFAC: bias solve failed (%s) — using raw gradient.", e)
                nb = module.bias.grad.float()
            self._update_param(module.bias, nb, lr, weight_decay, 0.0)

    @torch.no_grad()
    def step(self, closure=None):
        t_total = time.perf_counter()
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._step_count += 1
        self.hooks.flush()
        if should_refresh(self._step_count, self.factor_update_freq):
            self._update_factors()
        t_pre = time.perf_counter()
        todo = []
        for module in self.hooks.linear_layers:
            if module.weight.grad is None:
                continue
            lr, wd, mom = self._get_module_hp(module)
            if lr is None:
                continue
            todo.append((module, lr, wd, mom))
        nats = self._batched_natgrads([m for m, _, _, _ in todo])
        for module, lr, wd, mom in todo:
            self._apply_preconditioner(module, lr, wd, mom, nats.get(module))
        self.timing["precondition"].append(time.perf_counter() - t_pre)
        self.timing["total_step"].append(time.perf_counter() - t_total)
        return loss

    def get_timing_stats(self):
        stats = {}
        for key, times in self.timing.items():
            if times:
                arr = np.array(list(times))
                stats[key] = {"mean_ms": float(arr.mean() * 1000), "p50_ms": float(np.percentile(arr, 50) * 1000),
                              "p99_ms": float(np.percentile(arr, 99) * 1000), "total_s": float(arr.sum()),
                              "count": len(times)}
        return stats

    def capture(self):
        return self.hooks.capture()

    def pause_capture(self):
        self.hooks.pause()

    def resume_capture(self):
        self.hooks.resume()

    def cleanup(self):
        self.hooks.remove()
        self._factors.clear()
        self._classic_fallback.clear()
        self._momentum_buffers.clear()

    def __repr__(self) -> str:
        return (f"IFKFAC(damping={self.damping}, factor_update_freq={self.factor_update_freq}, "
                f"gamma={self.gamma}, augment_bias={self.augment_bias}, "
                f"n_layers={len(self.hooks.linear_layers)})")
