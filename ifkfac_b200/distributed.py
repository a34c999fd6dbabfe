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


def fold_merge(R_a: torch.Tensor, rows_a: int, R_b: torch.Tensor, rows_b: int, prec: int = 0) -> int:
    """[R_a; R_b] -> R_a on the device: the rows of R_b folded into R_a
    (precision mode ``prec``, ``_lib.PREC_*``).  A trapezoidal R_b (rows_b < n)
    is folded whole: exactly dependent columns (zero pivots) can leave some of
    its content below row rows_b.  The merged factor has min(n, rows_a + rows_b)
    meaningful rows."""
    n = R_a.shape[1]
    if min(rows_b, n) == 0:
        return rows_a
    triangular.fold_(R_a, rows_a, R_b, prec=prec, trapezoidal_chunk=True)
    return min(n, rows_a + rows_b)


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


class DistributedIFKFAC:
    """Data-parallel IFKFAC over a process group: the reference optimizer's
    semantics on the rows of every rank: the TSQR is sharded by batch rows, the
    local factors are combined by the merge tree of the reference's ``tsqr``
    (``ifkfac/triangular.py:150-227``), and whole layers are dealt to ranks for
    their solves.

    * Each rank's hooks fold that rank's rows (batch-sharded streaming TSQR).
    * At a refresh every layer's running factors are merged across ranks by the
      R-tree (:func:`rtree_merge`, the merge order of ``ifkfac/triangular.py:207-220``),
      so every rank finalizes the factors of all rows (and the row counts of all
      ranks scale them).
    * Gradients of the preconditioned layers are averaged across ranks (one
      ``all_reduce`` of a flat buffer) unless ``average_gradients=False`` (the
      caller already averages, e.g. under DDP).
    * The back-propagated rows δ a rank's hooks capture are those of that rank's
      loss.  With the usual loss, a mean over the rank's shard of a batch split in
      equal shards, each row is ``world`` times the row of the full-batch mean, so
      the merged R_G is scaled by ``delta_scale`` (default 1 / world; pass 1.0
      when each rank's loss is already normalised by the global batch).
    * Layer l's natural gradient and update run on rank ``l mod world`` only (its
      momentum buffer lives there); the owner then broadcasts the layer's
      parameters to the other ranks.

    Construct it on every rank with the same model and arguments; ``step()`` is a
    collective."""

    def __init__(self, model, *args, group: Optional[dist.ProcessGroup] = None,
                 average_gradients: bool = True, delta_scale: Optional[float] = None, **kwargs):
        from .ifkfac import IFKFAC
        self.opt = IFKFAC(model, *args, **kwargs)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.average_gradients = average_gradients
        self.delta_scale = 1.0 / self.world if delta_scale is None else float(delta_scale)
        self.owner = {m: i % self.world for i, m in enumerate(self.opt.hooks.linear_layers)}

    def __getattr__(self, name):
        return getattr(self.opt, name)

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.opt.zero_grad(set_to_none=set_to_none)

    def _merge_factors(self) -> None:
        h = self.opt.hooks
        if h.deferred:
            h._drain_deferred()
        layers = h.linear_layers
        dev = next(iter(self.opt.model.parameters())).device
        # every rank must take the same merges: agree first on each factor's width
        mine = torch.tensor([[0 if t[m] is None else t[m].n for t in (h._fx, h._fg)] for m in layers],
                            dtype=torch.int64, device=dev)
        allw = torch.empty(self.world, *mine.shape, dtype=torch.int64, device=dev)
        dist.all_gather(list(allw.unbind(0)), mine, group=self.group)
        width = allw.max(0).values.cpu().tolist()
        from .engine import Factor
        for li, m in enumerate(layers):
            for ti, (table, nrows) in enumerate(((h._fx, h._n_rows_X), (h._fg, h._n_rows_G))):
                n = int(width[li][ti])
                if n == 0:
                    continue  # no rank saw rows for this factor
                f = table[m]
                if f is None:
                    f = table[m] = Factor(n, dev, h.precision)
                rows, total = rtree_merge(f.R, f.rows_R, f.rows_seen, self.group,
                                          merge=lambda a, ra, b, rb, p=f.prec: fold_merge(a, ra, b, rb, p))
                f.rows_R, f.rows_seen = rows, total
                nrows[m] = total
                if ti == 1 and self.delta_scale != 1.0:
                    f.R.mul_(self.delta_scale)  # R^T R scales with the square of the rows

    def _average_gradients(self, params) -> None:
        grads = [p.grad for p in params if p.grad is not None]
        if not grads:
            return
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        dist.all_reduce(flat, group=self.group)
        flat /= self.world
        off = 0
        for g in grads:
            k = g.numel()
            g.copy_(flat[off:off + k].view_as(g))
            off += k

    @torch.no_grad()
    def step(self, closure=None):
        from .ifkfac import should_refresh
        opt = self.opt
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        opt._step_count += 1
        opt.hooks.flush()
        layers = [m for m in opt.hooks.linear_layers if m.weight.grad is not None]
        if self.average_gradients:
            self._average_gradients([p for m in layers for p in m.parameters()])
        if should_refresh(opt._step_count, opt.factor_update_freq):
            self._merge_factors()
            opt._update_factors()
        todo = []
        for m in layers:
            lr, wd, mom = opt._get_module_hp(m)
            if lr is not None and self.owner[m] == self.rank:
                todo.append((m, lr, wd, mom))
        nats = opt._batched_natgrads([m for m, _, _, _ in todo])
        for m, lr, wd, mom in todo:
            opt._apply_preconditioner(m, lr, wd, mom, nats.get(m))
        # the owners' updated parameters go to every rank
        for m in layers:
            for p in m.parameters():
                dist.broadcast(p.data, src=dist.get_global_rank(self.group, self.owner[m])
                               if self.group is not None else self.owner[m], group=self.group)
        return loss
