"""Batch-sharded streaming TSQR across data-parallel ranks.

Each rank folds its own share of the rows into a local running factor (the
hooks or :class:`ifkfac_b200.triangular.RunningFactor`).  :func:`rtree_merge`
then combines the local factors into the factor of all rows:

1. one ``all_gather`` of the local n x n factors (fp32, missing rows zero, into
   one stacked buffer) and one of their row counts;
2. the binary merge tree of the reference's ``tsqr``
   (``ifkfac/triangular.py:207-220``): round by round, adjacent pairs in rank
   order are merged, the odd one out is carried forward.  A merge folds the
   second factor's rows into the first as a trapezoidal chunk
   (``ifk_tsqr_fold`` with ``IFK_FOLD_TRAPEZOIDAL_CHUNK``, the structured
   [R_i; R_j] QR), which keeps the diagonal non-negative like the reference's
   sign normalisation.

Every rank runs the same tree over the same gathered inputs with the same
kernels, so every rank ends with the same factor.  The total row count (for the
1 / sqrt(p) scaling of ``get_factors``) is the sum over ranks.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import triangular

# merge(R_a, rows_a, R_b, rows_b) -> rows of the merged factor, written into R_a
Merge = Callable[[torch.Tensor, int, torch.Tensor, int], int]


def fold_merge(R_a: torch.Tensor, rows_a: int, R_b: torch.Tensor, rows_b: int) -> int:
    """[R_a; R_b] -> R_a on the device: the meaningful rows of R_b folded into R_a."""
    n = R_a.shape[1]
    k = min(rows_b, n)
    if k == 0:
        return rows_a
    return triangular.fold_(R_a, rows_a, R_b[:k], trapezoidal_chunk=True)


def tree_merge(factors: Sequence[torch.Tensor], rows: Sequence[int],
               merge: Merge = fold_merge) -> Tuple[torch.Tensor, int]:
    """Merge factors in the order of the reference ``tsqr`` tree; returns the
    surviving buffer (one of ``factors``, updated in place) and its row count."""
    if len(factors) != len(rows) or not factors:
        raise ValueError("tree_merge needs one row count per factor")
    items: List[Tuple[torch.Tensor, int]] = list(zip(factors, [int(r) for r in rows]))
    while len(items) > 1:
        merged = []
        for i in range(0, len(items), 2):
            if i + 1 < len(items):
                (ra, na), (rb, nb) = items[i], items[i + 1]
                merged.append((ra, merge(ra, na, rb, nb)))
            else:
                merged.append(items[i])  # odd one out: carried forward
        items = merged
    return items[0]


def gather_factors(R: torch.Tensor, rows: int, rows_seen: int,
                   group: Optional[dist.ProcessGroup] = None
                   ) -> Tuple[List[torch.Tensor], List[int], List[int]]:
    """All ranks' factors (views of one gathered tensor), meaningful row counts
    and total row counts, in rank order."""
    world = dist.get_world_size(group)
    n = R.shape[1]
    counts = torch.tensor([int(rows), int(rows_seen)], dtype=torch.int64, device=R.device)
    all_counts = torch.empty(world, 2, dtype=torch.int64, device=R.device)
    dist.all_gather(list(all_counts.unbind(0)), counts, group=group)
    stacked = torch.empty(world, n, n, dtype=R.dtype, device=R.device)
    factors = list(stacked.unbind(0))
    dist.all_gather(factors, R.contiguous(), group=group)
    c = all_counts.cpu().tolist()
    return factors, [r for r, _ in c], [s for _, s in c]


def rtree_merge(R: torch.Tensor, rows: int, rows_seen: int,
                group: Optional[dist.ProcessGroup] = None,
                merge: Merge = fold_merge) -> Tuple[int, int]:
    """Replace the local factor ``R`` (n x n fp32, ``rows`` meaningful rows,
    built from ``rows_seen`` data rows) by the factor of every rank's rows.
    Returns (meaningful rows, total data rows), identical on every rank."""
    if R.dim() != 2 or R.shape[0] != R.shape[1]:
        raise ValueError("rtree_merge expects an n x n factor buffer")
    factors, rows_all, seen_all = gather_factors(R, rows, rows_seen, group)
    merged, merged_rows = tree_merge(factors, rows_all, merge)
    R.copy_(merged)
    return merged_rows, sum(seen_all)


def merge_running(factor: triangular.RunningFactor,
                  group: Optional[dist.ProcessGroup] = None) -> None:
    """rtree_merge on a RunningFactor, in place (R, rows_R and rows_seen)."""
    factor.rows_R, factor.rows_seen = rtree_merge(factor.R, factor.rows_R, factor.rows_seen, group)
