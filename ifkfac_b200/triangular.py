"""Device-side curvature operations with the reference's functional API.

Same names and argument meaning as the reference's ``ifkfac/triangular.py``
(streaming_tsqr_update, batched_streaming_tsqr_update, finalize_R, tsqr,
apply_vered, apply_vered_batched, apply_vered_bias), computed by libifk.so on
CUDA tensors.  Differences that follow from the device library:

* factors are always fp32 (bf16 where the caller casts them); a bf16 chunk is
  accepted natively (the reference's geqrf has no bf16 kernel);
* every call requires CUDA tensors and raises otherwise: there is no CPU path.

``RunningFactor`` is the in-place accumulator the hooks use: an n x n fp32
buffer that stays on the device and absorbs chunks without reallocation.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib
from ._lib import check

__all__ = [
    "RunningFactor", "streaming_tsqr_update", "batched_streaming_tsqr_update", "finalize_R",
    "tsqr", "apply_vered", "apply_vered_batched", "apply_vered_bias", "damped_factor",
]

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"ifkfac_b200 supports float32 and bfloat16 tensors, got {t.dtype}") from None


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("ifkfac_b200 operates on CUDA tensors only (no CPU path)")


def _rows_contig(t: torch.Tensor) -> torch.Tensor:
    """Row-major with unit column stride (leading dimension = stride(0))."""
    if t.dim() != 2 or t.stride(1) != 1 or t.stride(0) < t.shape[1]:
        t = t.contiguous()
    return t


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def fold_(R: torch.Tensor, rows_R: int, chunk: torch.Tensor, prec: int = _lib.PREC_AUTO,
          trapezoidal_chunk: bool = False, status: Optional[torch.Tensor] = None) -> int:
    """Fold ``chunk`` into the n x n fp32 buffer ``R`` holding ``rows_R`` rows, in
    place.  Returns the new number of meaningful rows, min(n, rows_R + rows)."""
    _need_cuda(R, chunk)
    n = R.shape[1]
    if R.dtype != torch.float32 or R.shape != (n, n) or R.stride(1) != 1:
        raise ValueError("R must be an n x n row-major float32 buffer")
    chunk = _rows_contig(chunk)
    p = chunk.shape[0]
    if chunk.shape[1] != n:
        raise ValueError(f"chunk has {chunk.shape[1]} columns, factor has {n}")
    if p == 0:
        return rows_R
    L = _lib.lib()
    ws = _workspace(L.ifk_tsqr_fold_workspace(p, n), R.device)
    flags = _lib.FOLD_TRAPEZOIDAL_CHUNK if trapezoidal_chunk else 0
    sp = status.data_ptr() if status is not None else None
    check(L.ifk_tsqr_fold(R.data_ptr(), R.stride(0), rows_R, chunk.data_ptr(), chunk.stride(0), p,
                          n, _code(chunk), prec, flags, sp, ws.data_ptr(), ws.numel(), _stream()),
          "ifk_tsqr_fold")
    return min(n, rows_R + p)


def damped_factor(R: torch.Tensor, rows_R: int, rows_total: float, damping: float,
                  out_dtype: torch.dtype = torch.float32, prec: int = _lib.PREC_AUTO,
                  status: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """finalize_R(R / sqrt(rows_total), damping) cast to ``out_dtype``; None when
    the factor is still trapezoidal (rows_R < n), the reference's skip."""
    _need_cuda(R)
    n = R.shape[1]
    if rows_R < n:
        return None
    out = torch.empty(n, n, dtype=out_dtype, device=R.device)
    L = _lib.lib()
    ws = _workspace(L.ifk_finalize_workspace(n), R.device)
    sp = status.data_ptr() if status is not None else None
    check(L.ifk_finalize(R.data_ptr(), R.stride(0), rows_R, n, float(rows_total), float(damping),
                         out.data_ptr(), out.stride(0), _code(out), prec, sp, ws.data_ptr(),
                         ws.numel(), _stream()), "ifk_finalize")
    return out


class RunningFactor:
    """Running R of one Kronecker factor (n x n fp32 on the device) and its row counts."""

    __slots__ = ("n", "R", "rows_R", "rows_seen", "prec")

    def __init__(self, n: int, device, prec: int = _lib.PREC_AUTO):
        self.n = n
        self.R = torch.zeros(n, n, dtype=torch.float32, device=device)
        self.rows_R = 0
        self.rows_seen = 0
        self.prec = prec

    def fold(self, chunk: torch.Tensor) -> None:
        self.rows_R = fold_(self.R, self.rows_R, chunk, self.prec)
        self.rows_seen += chunk.shape[0]

    @property
    def value(self) -> torch.Tensor:
        """The reference's running R: shape (min(rows, n), n)."""
        return self.R[: self.rows_R]

    def damped(self, damping: float, out_dtype=torch.float32, status=None):
        return damped_factor(self.R, self.rows_R, self.rows_seen, damping, out_dtype,
                             _lib.PREC_BF16 if out_dtype == torch.bfloat16 else self.prec, status)

    def clear(self) -> None:
        self.R.zero_()
        self.rows_R = 0
        self.rows_seen = 0


def streaming_tsqr_update(running_R: Optional[torch.Tensor], new_chunk: torch.Tensor,
                          prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """Fold one chunk into the running R (reference: ifkfac/triangular.py:246-307).

    Returns an fp32 upper-trapezoidal R of shape (min(rows_so_far, n), n) with
    a non-negative diagonal, like the reference's leaf + merge QR."""
    _need_cuda(new_chunk)
    p, n = new_chunk.shape
    R = torch.zeros(n, n, dtype=torch.float32, device=new_chunk.device)
    rows_R = 0
    if running_R is not None:
        rows_R = running_R.shape[0]
        R[:rows_R] = running_R
    rows = fold_(R, rows_R, new_chunk, prec)
    return R[:rows]


def batched_streaming_tsqr_update(running_R: torch.Tensor, new_chunks: torch.Tensor,
                                  prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """(B, n, n) running factors (zeros for empty ones) and (B, p, n) zero-padded
    chunks (reference: ifkfac/triangular.py:331-379)."""
    B, p, n = new_chunks.shape
    out = running_R.to(torch.float32).clone()
    for b in range(B):
        fold_(out[b], n, new_chunks[b], prec)
    return out


def finalize_R(running_R: torch.Tensor, damping: float, prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """R of [R; sqrt(damping) I] with a non-negative diagonal (reference:
    ifkfac/triangular.py:386-421).  ``running_R`` must be square."""
    n = running_R.shape[1]
    if running_R.shape[0] != n:
        raise ValueError("finalize_R needs a square factor")
    R = _rows_contig(running_R.to(torch.float32))
    return damped_factor(R, n, 1.0, damping, torch.float32, prec)


def tsqr(M: torch.Tensor, tile_size: int = 512, prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """R factor of M (p >= n), non-negative diagonal (reference: ifkfac/triangular.py:150-227).

    The tile size of the reference's tree only changes rounding; the device
    fold streams sub-tiles of its own size."""
    p, n = M.shape
    if p < n:
        raise ValueError(f"tsqr requires p >= n (got p={p}, n={n})")
    return streaming_tsqr_update(None, M, prec)


def apply_vered(grad_W: torch.Tensor, R_X: torch.Tensor, R_G: torch.Tensor,
                prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """Natural gradient R_G^-1 R_G^-T grad_W R_X^-1 R_X^-T by four triangular
    solves (reference: ifkfac/triangular.py:551-656).  bf16-stored factors are
    read as bf16 (the reference upcasts them, :607-628); a non-square bf16 factor
    returns grad_W, as the reference does."""
    _need_cuda(grad_W, R_X, R_G)
    if R_X.dtype == torch.bfloat16 or R_G.dtype == torch.bfloat16:
        if R_X.shape[0] != R_X.shape[1] or R_G.shape[0] != R_G.shape[1]:
            return grad_W
    if R_X.dtype != R_G.dtype:
        R_X, R_G = R_X.float(), R_G.float()
    n_out, n_in = grad_W.shape
    if R_X.shape != (n_in, n_in) or R_G.shape != (n_out, n_out):
        raise ValueError("factor shapes do not match the gradient")
    g = _rows_contig(grad_W.to(torch.float32))
    R_X, R_G = _rows_contig(R_X), _rows_contig(R_G)
    nat = torch.empty(n_out, n_in, dtype=torch.float32, device=grad_W.device)
    L = _lib.lib()
    ws = _workspace(L.ifk_natgrad_workspace(n_out, n_in), grad_W.device)
    check(L.ifk_natgrad(g.data_ptr(), g.stride(0), R_X.data_ptr(), R_X.stride(0), R_G.data_ptr(),
                        R_G.stride(0), _code(R_X), nat.data_ptr(), nat.stride(0), n_out, n_in, prec,
                        None, ws.data_ptr(), ws.numel(), _stream()), "ifk_natgrad")
    return nat.to(grad_W.dtype) if grad_W.dtype != torch.float32 else nat


def apply_vered_batched(grad_W: torch.Tensor, R_X: torch.Tensor, R_G: torch.Tensor,
                        prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """Batched apply (reference: ifkfac/triangular.py:506-544)."""
    return torch.stack([apply_vered(grad_W[i], R_X[i], R_G[i], prec)
                        for i in range(grad_W.shape[0])], 0)


def apply_vered_bias(grad_b: torch.Tensor, R_G: torch.Tensor,
                     prec: int = _lib.PREC_AUTO) -> torch.Tensor:
    """R_G^-1 R_G^-T grad_b (reference: ifkfac/triangular.py:659-705)."""
    _need_cuda(grad_b, R_G)
    if R_G.dtype == torch.bfloat16 and R_G.shape[0] != R_G.shape[1]:
        return grad_b
    n = grad_b.shape[0]
    gb = grad_b.to(torch.float32).contiguous()
    R_G = _rows_contig(R_G)
    out = torch.empty(n, dtype=torch.float32, device=grad_b.device)
    L = _lib.lib()
    ws = _workspace(256, grad_b.device)
    check(L.ifk_natgrad_bias(gb.data_ptr(), R_G.data_ptr(), R_G.stride(0), _code(R_G),
                             out.data_ptr(), n, prec, ws.data_ptr(), ws.numel(), _stream()),
          "ifk_natgrad_bias")
    return out.to(grad_b.dtype) if grad_b.dtype != torch.float32 else out


def precond_update_(W: torch.Tensor, buf: Optional[torch.Tensor], nat: torch.Tensor, lr: float,
                    momentum: float, weight_decay: float, grad_clip: Optional[float],
                    buf_is_new: bool) -> None:
    """In-place epilogue (reference: ifkfac/ifkfac.py:394-413)."""
    _need_cuda(W, nat)
    if W.dtype != torch.float32 or nat.dtype != torch.float32 or not W.is_contiguous() \
            or not nat.is_contiguous():
        raise ValueError("update needs contiguous float32 W and nat")
    L = _lib.lib()
    ws = _workspace(L.ifk_update_workspace(W.numel()), W.device) if grad_clip else None
    check(L.ifk_update(W.data_ptr(), buf.data_ptr() if buf is not None else None, nat.data_ptr(),
                       W.numel(), float(lr), float(momentum), float(weight_decay),
                       float(grad_clip) if grad_clip else 0.0, 1 if buf_is_new else 0,
                       ws.data_ptr() if ws is not None else None,
                       ws.numel() if ws is not None else 0, _stream()), "ifk_update")


def bias_update_(b: torch.Tensor, nat_b: torch.Tensor, lr: float, weight_decay: float) -> None:
    """b *= 1 - lr*wd (wd > 0); b -= lr*nat_b (reference: ifkfac/ifkfac.py:415-423)."""
    _need_cuda(b, nat_b)
    L = _lib.lib()
    check(L.ifk_update_bias(b.data_ptr(), nat_b.contiguous().data_ptr(), b.numel(), float(lr),
                            float(weight_decay), _stream()), "ifk_update_bias")


def sqrt_rows(rows: int) -> float:
    return math.sqrt(rows)
