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
import math
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
        self.consumed = False  # R holds a damped factor (fused refresh) until clear()
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
        if self.consumed:
            raise RuntimeError("factor was consumed by a fused refresh; clear() it first")
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
        self.consumed = False


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
        if f.consumed:
            raise RuntimeError("factor was consumed by a fused refresh; clear() it first")
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


class Rows:
    """Rows of a 2-D device tensor for a fold, read in place by the fold kernels:
    ``x[index]`` (``index`` an int64 device tensor, or None for every row), with a
    column of ones appended when ``ones`` (the augmented-bias column).  The
    reference's hooks copy both (``ifkfac/activation_hooks.py:531-543``).

    :meth:`conv2d` gives the im2col rows of a Conv2d input (an NCHW tensor) the
    same way: the fold gathers each element from the image, so the
    ``F.unfold`` matrix of ``ifkfac/activation_hooks.py:489-499`` is never formed."""

    def __init__(self, x: torch.Tensor, index: Optional[torch.Tensor] = None, ones: bool = False):
        if x.dim() != 2:
            raise ValueError(f"Rows needs a 2-D tensor, got shape {tuple(x.shape)}")
        if x.dtype not in _DT:
            x = x.float()
        if x.stride(1) != 1:
            x = x.contiguous()
        if index is not None:
            index = index.to(device=x.device, dtype=torch.int64).contiguous()
            if index.dim() != 1:
                raise ValueError("Rows index must be 1-D")
        self.x, self.index, self.ones = x, index, bool(ones)
        self.geo = None  # im2col geometry (conv2d rows)

    @classmethod
    def conv2d(cls, x: torch.Tensor, module, index: Optional[torch.Tensor] = None) -> "Rows":
        """im2col rows (B * Ho * Wo, C * kh * kw) of the NCHW input ``x`` of the Conv2d
        ``module`` (F.unfold's order), optionally the rows ``index`` of them."""
        if x.dim() != 4:
            raise ValueError(f"a Conv2d input is N x C x H x W, got shape {tuple(x.shape)}")
        if x.dtype not in _DT:
            x = x.float()
        x = x.contiguous()
        r = cls.__new__(cls)
        pair = lambda v: (v, v) if isinstance(v, int) else tuple(v)
        (kh, kw), (sh, sw), (ph, pw), (dh, dw) = (pair(module.kernel_size), pair(module.stride),
                                                  pair(module.padding), pair(module.dilation))
        if isinstance(module.padding, str):
            raise ValueError("string padding is not supported by the im2col rows")
        B, C, H, W = x.shape
        Ho = (H + 2 * ph - dh * (kh - 1) - 1) // sh + 1
        Wo = (W + 2 * pw - dw * (kw - 1) - 1) // sw + 1
        r.x = x
        r.index = index.to(device=x.device, dtype=torch.int64).contiguous() if index is not None else None
        r.ones = False
        r.geo = dict(B=B, C=C, H=H, W=W, kh=kh, kw=kw, sh=sh, sw=sw, ph=ph, pw=pw, dh=dh, dw=dw, Ho=Ho, Wo=Wo)
        r._module = module
        return r

    @property
    def src_rows(self) -> int:
        if self.geo is not None:
            return self.geo["B"] * self.geo["Ho"] * self.geo["Wo"]
        return int(self.x.shape[0])

    @property
    def rows(self) -> int:
        return int(self.index.numel()) if self.index is not None else self.src_rows

    @property
    def cols(self) -> int:
        if self.geo is not None:
            return self.geo["C"] * self.geo["kh"] * self.geo["kw"]
        return int(self.x.shape[1]) + (1 if self.ones else 0)

    @property
    def dtype(self) -> torch.dtype:
        return self.x.dtype

    @property
    def device(self) -> torch.device:
        return self.x.device

    def conv_struct(self):
        g = self.geo
        return _lib.Conv2d(g["B"], g["C"], g["H"], g["W"], g["kh"], g["kw"], g["sh"], g["sw"],
                           g["ph"], g["pw"], g["dh"], g["dw"])

    def materialize(self) -> torch.Tensor:
        """The rows as a tensor of their own (what the reference's hooks build)."""
        if self.geo is not None:
            g = self.geo
            y = torch.nn.functional.unfold(self.x, kernel_size=(g["kh"], g["kw"]), dilation=(g["dh"], g["dw"]),
                                           padding=(g["ph"], g["pw"]), stride=(g["sh"], g["sw"]))
            y = y.permute(0, 2, 1).reshape(-1, self.cols)
            return y[self.index] if self.index is not None else y
        y = self.x[self.index] if self.index is not None else self.x
        if self.ones:
            y = torch.cat([y, torch.ones(y.shape[0], 1, device=y.device, dtype=y.dtype)], dim=1)
        return y


def as_rows(c) -> Rows:
    return c if isinstance(c, Rows) else Rows(c)


def fold_segments(factors: Sequence[Factor], segments: Sequence[Sequence], ws: torch.Tensor,
                  ident_tail: Optional[Sequence[float]] = None) -> torch.Tensor:
    """Fold the chunks segments[i] (tensors or :class:`Rows`) into factors[i] in
    order, without concatenating or gathering them: one persistent launch where
    they fit (ifk_tsqr_fold_segments), with the result of folding them one after
    another.  ident_tail[i] > 0 appends the rows ident_tail[i] * I (damping rows at
    the caller's scale); the factor then holds a damped factor and is marked
    consumed until clear().

    Returns the workspace actually used (grown if ``ws`` was too small)."""
    L = _lib.lib()
    segs, dts = [], set()
    for f, chunks in zip(factors, segments):
        if f.consumed:
            raise RuntimeError("factor was consumed by a fused refresh; clear() it first")
        cs = []
        for c in chunks:
            r = as_rows(c)
            if r.cols != f.n:
                raise ValueError(f"rows of width {r.cols} for a factor of width {f.n}")
            if r.rows == 0:
                continue
            cs.append(r)
            dts.add(r.dtype)
        segs.append(cs)
    precs = {f.prec for f in factors}
    if len(precs) > 1:
        raise ValueError("the factors of one segmented fold share a precision mode")
    if len(dts) > 1 and precs.pop() == _lib.PREC_AUTO:
        raise TypeError("with PREC_AUTO all chunks of a segmented fold share one dtype (the precision follows it)")
    dt = _DT[next(iter(dts))] if len(dts) == 1 else (_lib.PER_SEGMENT_DTYPE if dts else _lib.BF16)
    nf = len(factors)
    flat = [r for cs in segs for r in cs]
    arr = (_lib.Segment * max(len(flat), 1))()
    keep = []  # im2col geometries, alive for the call
    for i, r in enumerate(flat):
        if r.geo is not None:
            geo = r.conv_struct()
            keep.append(geo)
            arr[i] = _lib.Segment(r.x.data_ptr(), 0, r.rows, r.index.data_ptr() if r.index is not None else None,
                                  r.src_rows, r.cols, _DT[r.dtype], 0, ctypes.pointer(geo))
        else:
            arr[i] = _lib.Segment(r.x.data_ptr(), r.x.stride(0), r.rows,
                                  r.index.data_ptr() if r.index is not None else None, r.x.shape[0], r.x.shape[1],
                                  _DT[r.dtype], 0, None)
    ns = _arr(ctypes.c_int64, [f.n for f in factors])
    nseg = _arr(ctypes.c_int, [len(cs) for cs in segs])
    tail = _arr(ctypes.c_double, [float(v) for v in ident_tail]) if ident_tail is not None else None
    # fp32 mode: the workspace with which the segments share one wave schedule
    wsfn = (L.ifk_tsqr_fold_segments_fp32_workspace if factors[0].prec == _lib.PREC_FP32
            else L.ifk_tsqr_fold_segments_workspace)
    need = wsfn(nf, ns, nseg, arr, tail)
    if need == 0 and (flat or ident_tail):
        raise ValueError("ifk_tsqr_fold_segments_workspace rejected the shapes")
    if ws is None or ws.numel() < need:
        ws = _ws(need, factors[0].device)
    check(L.ifk_tsqr_fold_segments(
        nf, _arr(ctypes.c_void_p, [f.R.data_ptr() for f in factors]), ns,
        _arr(ctypes.c_int64, [f.rows_R for f in factors]), ns, nseg, arr, dt, tail, factors[0].prec,
        factors[0].status.data_ptr(), ws.data_ptr(), ws.numel(), _stream()), "ifk_tsqr_fold_segments")
    for i, (f, cs) in enumerate(zip(factors, segs)):
        p = sum(r.rows for r in cs)
        f.rows_R = min(f.n, f.rows_R + p)
        f.rows_seen += p
        if ident_tail is not None and ident_tail[i] > 0:
            f.consumed = True
    return ws


class LayerCurvature:
    """Device state of one layer's curvature path (factors, natgrad, momentum).

    ``window`` > 1 defers folding like the reference's deferred hook mode
    (``ifkfac/activation_hooks.py:347-364, 560-570``): chunks are kept (by
    reference; the caller keeps them alive) and folded ``window`` at a time in
    one persistent launch, in arrival order.  A full window is folded when the
    next chunk arrives or at the refresh, so the last one can share its launch
    with the damping rows (``refresh(consume=True)``); the factors are those of
    folding each chunk as it arrives."""

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
        # fold workspace of a full window (with the damping rows of a fused refresh)
        segs = (_lib.Segment * (2 * self.window))()
        for i in range(2 * self.window):
            segs[i] = _lib.Segment(None, 0, max(chunk_rows, 1), None, 0, 0)
        wsfn = (L.ifk_tsqr_fold_segments_fp32_workspace if self.fx.prec == _lib.PREC_FP32
                else L.ifk_tsqr_fold_segments_workspace)
        self.ws_pair = _ws(wsfn(
            2, _arr(ctypes.c_int64, [n_in, n_out]), _arr(ctypes.c_int, [self.window] * 2), segs,
            _arr(ctypes.c_double, [1.0, 1.0])), self.device)

    def fold(self, x_chunk: torch.Tensor, g_chunk: torch.Tensor) -> None:
        """Fold an activation chunk into R_X and a gradient chunk into R_G together
        (or keep them for a deferred fold when window > 1)."""
        if self.window <= 1:
            self.ws_pair = fold_batched((self.fx, self.fg), (x_chunk, g_chunk), self.ws_pair)
            return
        if self.fx.consumed:
            raise RuntimeError("factor was consumed by a fused refresh; clear() it first")
        if len(self._pending) >= self.window:
            self.flush()
        self._pending.append((x_chunk, g_chunk))

    def flush(self) -> None:
        """Fold the pending chunks (deferred mode): all of them in one launch per
        factor pair, in arrival order, without concatenating them."""
        if not self._pending:
            return
        segs = ([x for x, _ in self._pending], [g for _, g in self._pending])
        self._pending = []
        self.ws_pair = fold_segments((self.fx, self.fg), segs, self.ws_pair)

    # ---- factor refresh: get_factors + _update_factors (finite check, dtype) ----
    def refresh(self, damping: float, solve_prec: Optional[int] = None, consume: bool = False) -> bool:
        """Damped factors from the running R's; False (nothing queued) while either is
        still trapezoidal, the reference's per-layer skip (ifkfac/activation_hooks.py:287-300).

        consume=True is for a caller that clears the running factors after the
        refresh (the optimizer does after a successful get_factors,
        ifkfac/ifkfac.py:224-227): the
        pending chunks and the damping rows sqrt(damping * p) I are folded in the
        same launch into the running factors, which are then only good for clear();
        the damped factor is the result scaled by 1 / sqrt(p)."""
        fs, outs = (self.fx, self.fg), (self.RX, self.RG)
        pend = [sum(as_rows(c).rows for c in cs) for cs in zip(*self._pending)] if self._pending else [0, 0]
        square = all(min(f.n, f.rows_R + p) >= f.n for f, p in zip(fs, pend))
        fused = consume and damping > 0 and square
        if fused:
            segs = ([x for x, _ in self._pending], [g for _, g in self._pending])
            self._pending = []
            tails = [math.sqrt(damping * float(f.rows_seen + p)) for f, p in zip(fs, pend)]
            self.ws_pair = fold_segments(fs, segs, self.ws_pair, ident_tail=tails)
        else:
            self.flush()
        if self.fx.rows_R < self.n_in or self.fg.rows_R < self.n_out:
            return False
        L = _lib.lib()
        prec = self.prec if solve_prec is None else solve_prec
        check(L.ifk_finalize_batched(
            2, _arr(ctypes.c_void_p, [f.R.data_ptr() for f in fs]), _arr(ctypes.c_int64, [f.n for f in fs]),
            _arr(ctypes.c_int64, [f.rows_R for f in fs]), _arr(ctypes.c_int64, [f.n for f in fs]),
            _arr(ctypes.c_double, [float(f.rows_seen) for f in fs]), 0.0 if fused else float(damping),
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

    def natgrad_update(self, grad_W: torch.Tensor, W: torch.Tensor, lr: float, momentum: float,
                       weight_decay: float = 0.0) -> None:
        """The natural gradient and the update without clipping in one library call
        (ifk_natgrad_update).  Same result as :meth:`natgrad` followed by
        :meth:`update` with grad_clip None."""
        if grad_W.dtype != torch.float32 or grad_W.stride(1) != 1:
            grad_W = grad_W.float().contiguous()
        if not (W.is_contiguous() and W.dtype == torch.float32 and W.shape == (self.n_out, self.n_in)):
            raise ValueError("W must be a contiguous n_out x n_in float32 tensor")
        L = _lib.lib()
        p = self.prec
        if p == _lib.PREC_AUTO:
            p = _lib.PREC_BF16 if self.factor_dtype == torch.bfloat16 else _lib.PREC_FP32
        new_buf = False
        if momentum > 0 and self.buf is None:
            self.buf = torch.empty(self.n_out, self.n_in, dtype=torch.float32, device=self.device)
            new_buf = True
        need = L.ifk_natgrad_update_workspace(self.n_out, self.n_in)
        if getattr(self, "ws_ngu", None) is None or self.ws_ngu.numel() < need:
            self.ws_ngu = _ws(need, self.device)
        check(L.ifk_natgrad_update(
            grad_W.data_ptr(), grad_W.stride(0), self.RX.data_ptr(), self.n_in, self.RG.data_ptr(), self.n_out,
            _DT[self.factor_dtype], W.data_ptr(), self.buf.data_ptr() if momentum > 0 else None, self.n_out,
            self.n_in, float(lr), float(momentum), float(weight_decay), 1 if new_buf else 0, p,
            self.status.data_ptr(), self.ws_ngu.data_ptr(), self.ws_ngu.numel(), _stream()),
            "ifk_natgrad_update")

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
