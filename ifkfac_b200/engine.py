"""Per-layer curvature state on the device, with preallocated buffers.

``LayerCurvature`` holds everything one Linear layer needs on the hot path:
the running factors R_X (n_in x n_in) and R_G (n_out x n_out) in fp32, the
damped factors (fp32 or bf16), the natural-gradient buffer, the momentum
buffer and the libifk workspaces.  All buffers are allocated once, so a
training step issues only library calls on the current stream and can be
captured in a CUDA graph.  Row counts are host integers, as in the
reference's hooks (``_n_rows_X`` / ``_n_rows_G``, ifkfac/activation_hooks.py:205-206).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import check

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


class Factor:
    """One running Kronecker factor: R (n x n fp32), its row counts, its fold workspace."""

    def __init__(self, n: int, device, prec: int = _lib.PREC_AUTO, chunk_rows: int = 0):
        self.n = n
        self.device = torch.device(device)
        self.prec = prec
        self.R = torch.zeros(n, n, dtype=torch.float32, device=self.device)
        self.rows_R = 0
        self.rows_seen = 0
        self.ws = _ws(_lib.lib().ifk_tsqr_fold_workspace(max(chunk_rows, 1), n), self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def _ensure_ws(self, rows: int) -> None:
        need = _lib.lib().ifk_tsqr_fold_workspace(rows, self.n)
        if self.ws.numel() < need:
            self.ws = _ws(need, self.device)

    def fold(self, chunk: torch.Tensor, trapezoidal: bool = False) -> None:
        """R <- R of [R; chunk] (streaming_tsqr_update, ifkfac/triangular.py:246-307)."""
        if chunk.dim() != 2 or chunk.shape[1] != self.n:
            raise ValueError(f"chunk of shape {tuple(chunk.shape)} for a factor of width {self.n}")
        if chunk.stride(1) != 1:
            chunk = chunk.contiguous()
        p = chunk.shape[0]
        if p == 0:
            return
        self._ensure_ws(p)
        flags = _lib.FOLD_TRAPEZOIDAL_CHUNK if trapezoidal else 0
        check(_lib.lib().ifk_tsqr_fold(
            self.R.data_ptr(), self.n, self.rows_R, chunk.data_ptr(), chunk.stride(0), p, self.n,
            _DT[chunk.dtype], self.prec, flags, self.status.data_ptr(), self.ws.data_ptr(),
            self.ws.numel(), _stream()), "ifk_tsqr_fold")
        self.rows_R = min(self.n, self.rows_R + p)
        self.rows_seen += p

    def clear(self) -> None:
        self.R.zero_()
        self.rows_R = 0
        self.rows_seen = 0


def _arr(ctype, vals):
    return (ctype * len(vals))(*vals)


def fold_batched(factors: Sequence[Factor], chunks: Sequence[torch.Tensor], ws: torch.Tensor,
                 trapezoidal: bool = False) -> torch.Tensor:
    """Fold chunks[i] into factors[i], all in one wave schedule (ifk_tsqr_fold_batched).

    Returns the workspace actually used (grown if ``ws`` was too small)."""
    L = _lib.lib()
    cs = []
    for f, c in zip(factors, chunks):
        if c.dim() != 2 or c.shape[1] != f.n:
            raise ValueError(f"chunk of shape {tuple(c.shape)} for a factor of width {f.n}")
        cs.append(c if c.stride(1) == 1 else c.contiguous())
    dts = {c.dtype for c in cs}
    if len(dts) != 1:
        raise TypeError("all chunks of a batched fold must share one dtype")
    nf = len(factors)
    rows = _arr(ctypes.c_int64, [c.shape[0] for c in cs])
    ns = _arr(ctypes.c_int64, [f.n for f in factors])
    need = L.ifk_tsqr_fold_batched_workspace(nf, rows, ns)
    if ws is None or ws.numel() < need:
        ws = _ws(need, factors[0].device)
    check(L.ifk_tsqr_fold_batched(
        nf, _arr(ctypes.c_void_p, [f.R.data_ptr() for f in factors]), ns,
        _arr(ctypes.c_int64, [f.rows_R for f in factors]), _arr(ctypes.c_void_p, [c.data_ptr() for c in cs]),
        _arr(ctypes.c_int64, [c.stride(0) for c in cs]), rows, ns, _DT[cs[0].dtype], factors[0].prec,
        _lib.FOLD_TRAPEZOIDAL_CHUNK if trapezoidal else 0, factors[0].status.data_ptr(), ws.data_ptr(),
        ws.numel(), _stream()), "ifk_tsqr_fold_batched")
    for f, c in zip(factors, cs):
        f.rows_R = min(f.n, f.rows_R + c.shape[0])
        f.rows_seen += c.shape[0]
    return ws


def _rows_view(chunks: Sequence[torch.Tensor]) -> torch.Tensor:
    """The chunks stacked by rows: a view when they are consecutive row slices of
    one tensor (no copy), else a concatenation."""
    c0 = chunks[0]
    if len(chunks) == 1:
        return c0
    es, rs = c0.element_size(), c0.stride(0)
    adjacent = all(c.dtype == c0.dtype and c.shape[1] == c0.shape[1] and c.stride() == c0.stride()
                   and c.stride(1) == 1 and c.untyped_storage().data_ptr() == c0.untyped_storage().data_ptr()
                   for c in chunks)
    for a, b in zip(chunks, chunks[1:]):
        adjacent = adjacent and b.data_ptr() == a.data_ptr() + a.shape[0] * rs * es
    if adjacent:
        return torch.as_strided(c0, (sum(c.shape[0] for c in chunks), c0.shape[1]), c0.stride())
    return torch.cat(list(chunks), 0)


class LayerCurvature:
    """Device state of one layer's curvature path (factors, natgrad, momentum).

    ``window`` > 1 defers folding like the reference's deferred hook mode
    (``ifkfac/activation_hooks.py:347-364``): chunks are kept (by reference; the
    caller keeps them alive) until ``window`` of them are pending or the factors
    are refreshed, then folded as one chunk of all their rows, so one persistent
    launch covers several tiles."""

    def __init__(self, n_in: int, n_out: int, device, prec: int = _lib.PREC_AUTO,
                 factor_dtype: torch.dtype = torch.float32, chunk_rows: int = 0, window: int = 1):
        L = _lib.lib()
        self.window = max(int(window), 1)
        self._pending: List[Tuple[torch.Tensor, torch.Tensor]] = []
        self.n_in, self.n_out = n_in, n_out
        self.device = torch.device(device)
        self.prec = prec
        self.fx = Factor(n_in, device, prec, chunk_rows)
        self.fg = Factor(n_out, device, prec, chunk_rows)
        self.factor_dtype = factor_dtype
        self.RX = torch.empty(n_in, n_in, dtype=factor_dtype, device=self.device)
        self.RG = torch.empty(n_out, n_out, dtype=factor_dtype, device=self.device)
        self.have_factors = False
        self.ws_fin = _ws(L.ifk_finalize_batched_workspace(2, _arr(ctypes.c_int64, [n_in, n_out])),
                          self.device)
        self.ws_nat = _ws(L.ifk_natgrad_workspace(n_out, n_in), self.device)
        self.ws_upd = _ws(L.ifk_update_workspace(n_out * n_in), self.device)
        self.nat = torch.empty(n_out, n_in, dtype=torch.float32, device=self.device)
        self.buf: Optional[torch.Tensor] = None
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.fx.status = self.status
        self.fg.status = self.status
        rows = max(chunk_rows, 1) * self.window
        self.ws_pair = _ws(L.ifk_tsqr_fold_batched_workspace(
            2, _arr(ctypes.c_int64, [rows, rows]), _arr(ctypes.c_int64, [n_in, n_out])), self.device)

    def fold(self, x_chunk: torch.Tensor, g_chunk: torch.Tensor) -> None:
        """Fold an activation chunk into R_X and a gradient chunk into R_G together
        (or keep them for a deferred fold when window > 1)."""
        if self.window <= 1:
            self.ws_pair = fold_batched((self.fx, self.fg), (x_chunk, g_chunk), self.ws_pair)
            return
        self._pending.append((x_chunk, g_chunk))
        if len(self._pending) >= self.window:
            self.flush()

    def flush(self) -> None:
        """Fold the pending chunks (deferred mode) as one chunk per factor."""
        if not self._pending:
            return
        x = _rows_view([x for x, _ in self._pending])
        g = _rows_view([g for _, g in self._pending])
        self._pending = []
        self.ws_pair = fold_batched((self.fx, self.fg), (x, g), self.ws_pair)

    # ---- factor refresh: get_factors + _update_factors (finite check, dtype) ----
    def refresh(self, damping: float, solve_prec: Optional[int] = None) -> bool:
        """Damped factors from the running R's; False (nothing queued) while either is
        still trapezoidal, the reference's per-layer skip (ifkfac/activation_hooks.py:287-300)."""
        self.flush()
        if self.fx.rows_R < self.n_in or self.fg.rows_R < self.n_out:
            return False
        L = _lib.lib()
        prec = self.prec if solve_prec is None else solve_prec
        fs, outs = (self.fx, self.fg), (self.RX, self.RG)
        check(L.ifk_finalize_batched(
            2, _arr(ctypes.c_void_p, [f.R.data_ptr() for f in fs]), _arr(ctypes.c_int64, [f.n for f in fs]),
            _arr(ctypes.c_int64, [f.rows_R for f in fs]), _arr(ctypes.c_int64, [f.n for f in fs]),
            _arr(ctypes.c_double, [float(f.rows_seen) for f in fs]), float(damping),
            _arr(ctypes.c_void_p, [o.data_ptr() for o in outs]), _arr(ctypes.c_int64, [f.n for f in fs]),
            _DT[self.factor_dtype], prec, self.status.data_ptr(), self.ws_fin.data_ptr(),
            self.ws_fin.numel(), _stream()), "ifk_finalize_batched")
        self.have_factors = True
        return True

    def factors_finite(self) -> bool:
        """Reads the device status word (a sync), like torch.isfinite(R).all() in
        ifkfac/ifkfac.py:231-237."""
        st = int(self.status.item())
        if st == _lib.ERR_TIMEOUT:
            raise _lib.IFKError(st, "device wait")
        return st != _lib.ERR_NONFINITE

    def reset_status(self) -> None:
        self.status.zero_()

    # ---- natural gradient + update ----
    def natgrad(self, grad_W: torch.Tensor, prec: Optional[int] = None) -> torch.Tensor:
        """nat = R_G^-1 R_G^-T grad_W R_X^-1 R_X^-T (apply_vered, ifkfac/triangular.py:551-656)."""
        if grad_W.dtype != torch.float32 or grad_W.stride(1) != 1:
            grad_W = grad_W.float().contiguous()
        p = self.prec if prec is None else prec
        if p == _lib.PREC_AUTO:
            p = _lib.PREC_BF16 if self.factor_dtype == torch.bfloat16 else _lib.PREC_FP32
        check(_lib.lib().ifk_natgrad(
            grad_W.data_ptr(), grad_W.stride(0), self.RX.data_ptr(), self.n_in, self.RG.data_ptr(),
            self.n_out, _DT[self.factor_dtype], self.nat.data_ptr(), self.n_in, self.n_out,
            self.n_in, p, self.status.data_ptr(), self.ws_nat.data_ptr(), self.ws_nat.numel(),
            _stream()), "ifk_natgrad")
        return self.nat

    def update(self, W: torch.Tensor, nat: torch.Tensor, lr: float, momentum: float,
               weight_decay: float, grad_clip: Optional[float]) -> None:
        """Epilogue of ifkfac/ifkfac.py:394-413 on fp32 master weights, in place."""
        new_buf = False
        if momentum > 0 and self.buf is None:
            self.buf = torch.empty(self.n_out, self.n_in, dtype=torch.float32, device=self.device)
            new_buf = True
        check(_lib.lib().ifk_update(
            W.data_ptr(), self.buf.data_ptr() if momentum > 0 else None, nat.data_ptr(), W.numel(),
            float(lr), float(momentum), float(weight_decay), float(grad_clip or 0.0),
            1 if new_buf else 0, self.ws_upd.data_ptr(), self.ws_upd.numel(), _stream()),
            "ifk_update")

    def clear(self) -> None:
        self._pending = []
        self.fx.clear()
        self.fg.clear()
