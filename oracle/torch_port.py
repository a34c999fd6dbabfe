"""The reference's executed C2 path restated on torch CPU calls (TEST / BASELINE ONLY).

``oracle/ifk_oracle.py`` is the parity oracle (numpy + scipy LAPACK, R-only
``geqrf``).  This module is the CPU *baseline* of ``bench.py``: the same steps
through the same library calls the reference makes, so that the timed work is
the reference's own, including the explicit Q that ``torch.linalg.qr(...,
mode="reduced")`` forms and the reference then discards.  Only ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs and ``tests/`` may import it; the
product path never does.

Citations are ``path:line`` inside the reference project.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def positive_diagonal_R(R: torch.Tensor) -> torch.Tensor:
    """``ifkfac/triangular.py:230-239``: row i times sign(R[i, i]) (0 -> +1)."""
    s = torch.sign(torch.diagonal(R))
    s = torch.where(s == 0, torch.ones_like(s), s)
    return R * s.unsqueeze(1)


def streaming_tsqr_update(running_R: Optional[torch.Tensor], chunk: torch.Tensor) -> torch.Tensor:
    """``ifkfac/triangular.py:246-307``: leaf QR of the chunk (mode="reduced", :284),
    then the merge QR of [running_R; R_new] (:299-300), sign-normalised."""
    _, r_new = torch.linalg.qr(chunk, mode="reduced")
    if running_R is None:
        return positive_diagonal_R(r_new)
    _, r = torch.linalg.qr(torch.cat([running_R, r_new], dim=0), mode="reduced")
    return positive_diagonal_R(r)


def finalize_R(running_R: torch.Tensor, damping: float) -> torch.Tensor:
    """``ifkfac/triangular.py:386-421``: QR of [R; sqrt(damping) I], sign-normalised."""
    n = running_R.shape[0]
    damp = (damping ** 0.5) * torch.eye(n, dtype=running_R.dtype)
    _, r = torch.linalg.qr(torch.cat([running_R, damp], dim=0), mode="reduced")
    return positive_diagonal_R(r)


def get_factor(running_R: torch.Tensor, rows: int, damping: float) -> torch.Tensor:
    """One factor of ``get_factors`` (``ifkfac/activation_hooks.py:323-332``): R / sqrt(rows),
    then ``finalize_R``."""
    return finalize_R(running_R / math.sqrt(rows), damping)


def apply_vered_bf16_stored(grad_W: torch.Tensor, R_X: torch.Tensor, R_G: torch.Tensor) -> torch.Tensor:
    """``ifkfac/triangular.py:607-628``: factors stored in bf16 (use_true_bf16) are
    upcast to fp32 and the four solves run in fp32."""
    rx, rg, g = R_X.float(), R_G.float(), grad_W.float()
    t1 = torch.linalg.solve_triangular(rg.t(), g, upper=False)
    t2 = torch.linalg.solve_triangular(rg, t1, upper=True)
    t3 = torch.linalg.solve_triangular(rx.t(), t2.t(), upper=False)
    t4 = torch.linalg.solve_triangular(rx, t3, upper=True)
    return t4.t().contiguous()


def precond_update_(W: torch.Tensor, buf: Optional[torch.Tensor], nat: torch.Tensor, lr: float,
                    momentum: float) -> torch.Tensor:
    """``ifkfac/ifkfac.py:394-413`` without clip or decay: buf = mom * buf + nat
    (zero-initialised), W -= lr * buf.  Returns the buffer."""
    if buf is None:
        buf = torch.zeros_like(nat)
    buf.mul_(momentum).add_(nat)
    W.add_(buf, alpha=-lr)
    return buf
