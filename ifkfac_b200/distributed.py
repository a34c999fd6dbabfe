"""Batch-sharded streaming TSQR across data-parallel ranks.

Each rank folds its own share of the rows into a local running factor (the
hooks or :class:`ifkfac_b200.triangular.RunningFactor`).  :func:`rtree_merge`
then combines the local factors into the factor of all rows, in the merge
order of the reference's ``tsqr`` tree (``ifkfac/triangular.py:207-220``:
round by round, adjacent pairs in rank order, the odd one carried forward):

1. one small ``all_gather`` of the ranks' row counts, so that every rank knows
   the row count of every subtree;
2. ceil(log2 world) rounds of pairwise exchange: in the round of stride s, rank
   i (i mod 2s == 0) receives the factor of rank i + s and merges it into its
   own, and rank i + s leaves the tree.  The merges of one round run on
   different ranks at the same time.  A merge folds the second factor's rows
   into the first as a trapezoidal chunk (``ifk_tsqr_fold`` with
   ``IFK_FOLD_TRAPEZOIDAL_CHUNK``, the structured [R_i; R_j] QR), which keeps
   the diagonal non-negative like the reference's sign normalisation;
3. a broadcast of rank 0's merged factor.

So every rank ends with the same factor.  The total row count (for the
1 / sqrt(p) scaling of ``get_factors``) is the sum over ranks.
:func:`tree_merge` runs the same tree on factors that one process holds.
"""
from __future__ import annotations

import logging
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import triangular

logger = logging.getLogger(__name__)

# merge(R_a, rows_a, R_b, rows_b) -> rows of the merged factor, written into R_a
Merge = Callable[[torch.Tensor, int, torch.Tensor, int], int]


def fold_merge(R_a: torch.Tensor, rows_a: int, R_b: torch.Tensor, rows_b: int, prec: int = 0) -> int:
    """[R_a; R_b] -> R_a on the device: the rows of R_b folded into R_a
    (precision mode ``prec``, ``_lib.PREC_*``).  A trapezoidal R_b (rows_b < n)
    is folded whole: exactly dependent columns (zero pivots) can leave some of
    its content below row rows_b.  The merged factor has min(n, rows_a + rows_b)
    meaningful rows."""
    from . import _lib
    n = R_a.shape[1]
    if min(rows_b, n) == 0:
        return rows_a
    # bf16 mode keeps the rows past a factor's count zero (the fold's rank bound),
    # so only the meaningful rows are folded
    chunk = R_b[:min(rows_b, n)] if prec == _lib.PREC_BF16 else R_b
    triangular.fold_(R_a, rows_a, chunk, prec=prec, trapezoidal_chunk=True)
    return min(n, rows_a + rows_b)


def tree_merge_device(factors: Sequence[torch.Tensor], rows: Sequence[int], prec: int) -> int:
    """The tree of :func:`tree_merge` on factors one process holds, by the library's
    ``ifk_rtree_merge`` (the merges of each round in one launch); the result is in
    ``factors[0]``.  Returns its meaningful rows."""
    import ctypes
    from . import _lib
    L = _lib.lib()
    k = len(factors)
    if k != len(rows) or k == 0:
        raise ValueError("tree_merge_device needs one row count per factor")
    n = factors[0].shape[1]
    for f in factors:
        if f.dtype != torch.float32 or f.shape != (n, n) or f.stride(1) != 1 or not f.is_cuda:
            raise ValueError("factors must be n x n row-major float32 CUDA tensors")
    ws = torch.empty(max(int(L.ifk_rtree_merge_workspace(k, n)), 256), dtype=torch.uint8, device=factors[0].device)
    out = ctypes.c_int64(0)
    _lib.check(L.ifk_rtree_merge(
        k, (ctypes.c_void_p * k)(*[f.data_ptr() for f in factors]),
        (ctypes.c_int64 * k)(*[f.stride(0) for f in factors]), (ctypes.c_int64 * k)(*[int(r) for r in rows]),
        n, prec, ctypes.byref(out), None, ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream().cuda_stream), "ifk_rtree_merge")
    return int(out.value)


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


def _global_rank(group, r: int) -> int:
    return dist.get_global_rank(group, r) if group is not None else r


def rtree_merge(R: torch.Tensor, rows: int, rows_seen: int,
                group: Optional[dist.ProcessGroup] = None,
                merge: Merge = fold_merge) -> Tuple[int, int]:
    """Replace the local factor ``R`` (n x n fp32, ``rows`` meaningful rows,
    built from ``rows_seen`` data rows) by the factor of every rank's rows, by
    pairwise merges in ceil(log2 world) rounds and a broadcast (the tree of
    ``ifkfac/triangular.py:207-220``).  Returns (meaningful rows, total data
    rows), identical on every rank.  If a collective fails (a rank that never
    posts its factor makes its partner's receive time out), the error
    propagates and ``R`` is left as it was: the merges run on a copy."""
    if R.dim() != 2 or R.shape[0] != R.shape[1]:
        raise ValueError("rtree_merge expects an n x n factor buffer")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = R.shape[1]
    counts = torch.tensor([int(rows), int(rows_seen)], dtype=torch.int64, device=R.device)
    all_counts = torch.empty(world, 2, dtype=torch.int64, device=R.device)
    dist.all_gather(list(all_counts.unbind(0)), counts, group=group)
    c = all_counts.cpu().tolist()
    rows_all, seen_all = [r for r, _ in c], [x for _, x in c]
    total_rows, total_seen = min(n, sum(rows_all)), sum(seen_all)
    if world == 1:
        return total_rows, total_seen
    work = R.clone()
    cur = min(n, rows_all[rank])
    other = None
    s = 1
    while s < world:
        if rank % (2 * s) == 0:
            partner = rank + s
            if partner < world:
                rb = min(n, sum(rows_all[partner:partner + s]))
                if rb > 0:
                    if other is None:
                        other = torch.empty_like(work)
                    dist.recv(other, src=_global_rank(group, partner), group=group)
                    cur = merge(work, cur, other, rb)
        else:
            # rank % 2s == s: hand the subtree's factor to rank - s and leave the tree
            if cur > 0:
                dist.send(work, dst=_global_rank(group, rank - s), group=group)
            break
        s *= 2
    dist.broadcast(work, src=_global_rank(group, 0), group=group)
    R.copy_(work)
    return total_rows, total_seen


def merge_or_skip(R: torch.Tensor, rows: int, rows_seen: int,
                  group: Optional[dist.ProcessGroup] = None,
                  merge: Merge = fold_merge) -> Optional[Tuple[int, int]]:
    """:func:`rtree_merge`, or None with a warning when a collective of the merge
    failed (a peer never posted its factor and the process group's timeout ran
    out, or the peer is gone).  ``R`` is then unchanged, so the caller can keep
    its running factor and skip the factor update, as the reference does when a
    refresh cannot be computed (``ifkfac/ifkfac.py:207-223``)."""
    try:
        return rtree_merge(R, rows, rows_seen, group, merge)
    except (RuntimeError, dist.DistError) as e:  # timeouts and lost peers surface as these
        logger.warning("IFKFAC: R-tree merge failed (%s); factor update skipped", e)
        return None


# merge_many([(R_a, rows_a, R_b, rows_b, prec), ...]): each R_b's rows folded into
# its R_a, in place (R_b holds only the rows that are sent: rows_b of them in bf16
# mode, the whole factor in fp32 mode)
MergeMany = Callable[[Sequence[Tuple[torch.Tensor, int, torch.Tensor, int, int]]], None]


def fold_merge_many(jobs: Sequence[Tuple[torch.Tensor, int, torch.Tensor, int, int]]) -> None:
    """The merges of one round of :func:`rtree_reduce_many` on the device: the
    trapezoidal folds of each precision in one ``ifk_tsqr_fold_batched`` call
    (the library runs up to 64 of them per persistent launch)."""
    import ctypes
    from . import _lib
    from .engine import _arr, _stream
    L = _lib.lib()
    by_prec = {}
    for j in jobs:
        if j[2].shape[0] > 0:
            by_prec.setdefault(j[4], []).append(j)
    for prec, js in by_prec.items():
        k = len(js)
        ns = [ra.shape[1] for ra, _, _, _, _ in js]
        rows = [rb.shape[0] for _, _, rb, _, _ in js]
        dev = js[0][0].device
        need = int(L.ifk_tsqr_fold_batched_workspace(k, _arr(ctypes.c_int64, rows), _arr(ctypes.c_int64, ns)))
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.check(L.ifk_tsqr_fold_batched(
            k, _arr(ctypes.c_void_p, [ra.data_ptr() for ra, _, _, _, _ in js]),
            _arr(ctypes.c_int64, [ra.stride(0) for ra, _, _, _, _ in js]),
            _arr(ctypes.c_int64, [min(na, ra.shape[1]) for ra, na, _, _, _ in js]),
            _arr(ctypes.c_void_p, [rb.data_ptr() for _, _, rb, _, _ in js]),
            _arr(ctypes.c_int64, [rb.stride(0) for _, _, rb, _, _ in js]), _arr(ctypes.c_int64, rows),
            _arr(ctypes.c_int64, ns), _lib.F32, prec, _lib.FOLD_TRAPEZOIDAL_CHUNK, status.data_ptr(),
            ws.data_ptr(), ws.numel(), _stream()), "ifk_tsqr_fold_batched")


def rtree_reduce_many(items: Sequence[Tuple[torch.Tensor, int, int, int]], owners: Sequence[int],
                      group: Optional[dist.ProcessGroup] = None, merge_many: MergeMany = fold_merge_many,
                      bucket_bytes: int = 1 << 30) -> List[Tuple[int, int]]:
    """The R-tree of :func:`rtree_merge` for many factors at once, each reduced to
    its owner rank instead of to rank 0 and broadcast.

    ``items[f] = (R, rows, rows_seen, prec)``: this rank's local factor f (n x n
    fp32, ``rows`` meaningful rows, built from ``rows_seen`` data rows; ``prec``
    the fold precision, ``_lib.PREC_*``).  Factor f is merged over the ranks
    relabelled from ``owners[f]`` (relative rank (rank - owner) mod world), in the
    order of the reference's ``tsqr`` tree over the relative ranks
    (``ifkfac/triangular.py:207-220``: adjacent pairs, odd one carried forward),
    so that the factor of all rows ends in ``items[f][0]`` on the owner.  Other
    ranks' buffers hold partial merges or their local factor afterwards.

    One ``all_gather`` of every factor's counts; then per round of the tree, the
    exchanges of all factors go in buckets of at most ``bucket_bytes`` (a bucket
    is a run of consecutive factors, the same on every rank, so every pair of
    ranks posts its sends and receives in the same order) as one
    ``batch_isend_irecv`` each, and the bucket's merges as one batched fold.  In
    bf16 mode only the meaningful rows of a factor are sent (the fold keeps the
    rows past a factor's count zero); fp32 mode sends the whole factor, which is
    folded whole like :func:`fold_merge` does.

    Returns (meaningful rows, total data rows) of every merged factor, the same on
    every rank.  A failed collective raises; the buffers may then hold partial
    merges, so the caller drops them (``DistributedIFKFAC`` clears its running
    factors)."""
    from . import _lib
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    nf = len(items)
    if len(owners) != nf:
        raise ValueError("rtree_reduce_many needs one owner per factor")
    for R, _, _, _ in items:
        if R.dim() != 2 or R.shape[0] != R.shape[1] or not R.is_contiguous():
            raise ValueError("rtree_reduce_many expects contiguous n x n factor buffers")
    if nf == 0:
        return []
    dev = items[0][0].device
    ns = [R.shape[1] for R, _, _, _ in items]
    counts = torch.tensor([[min(n, int(r)), int(s)] for n, (_, r, s, _) in zip(ns, items)],
                          dtype=torch.int64, device=dev)
    allc = torch.empty(world, nf, 2, dtype=torch.int64, device=dev)
    dist.all_gather(list(allc.unbind(0)), counts, group=group)
    c = allc.cpu().tolist()  # c[rank][factor] = [rows, rows_seen]
    results = [(min(ns[f], sum(c[q][f][0] for q in range(world))), sum(c[q][f][1] for q in range(world)))
               for f in range(nf)]
    if world == 1:
        return results
    cur = [min(ns[f], c[rank][f][0]) for f in range(nf)]
    active = [True] * nf
    # buckets: runs of consecutive factors of at most bucket_bytes (the same on every rank)
    buckets, lo, acc = [], 0, 0
    for f in range(nf):
        b = ns[f] * ns[f] * 4
        if f > lo and acc + b > bucket_bytes:
            buckets.append((lo, f))
            lo, acc = f, 0
        acc += b
    buckets.append((lo, nf))
    s = 1
    while s < world:
        plan = [None] * nf  # ('recv', partner, rows_b) or ('send', dst)
        for f in range(nf):
            if not active[f]:
                continue
            rel = (rank - owners[f]) % world
            if rel % (2 * s) == 0:
                prel = rel + s
                if prel < world:
                    rb = min(ns[f], sum(c[(owners[f] + q) % world][f][0] for q in range(prel, min(world, prel + s))))
                    if rb > 0:
                        plan[f] = ("recv", (owners[f] + prel) % world, rb)
            else:  # rel mod 2s == s: hand the subtree's factor on and leave the tree
                active[f] = False
                if cur[f] > 0:
                    plan[f] = ("send", (owners[f] + rel - s) % world)
        for lo, hi in buckets:
            ops, jobs = [], []
            for f in range(lo, hi):
                p = plan[f]
                if p is None:
                    continue
                R, _, _, prec = items[f]
                if p[0] == "recv":
                    nrows = p[2] if prec == _lib.PREC_BF16 else ns[f]
                    buf = torch.empty(nrows, ns[f], dtype=R.dtype, device=dev)
                    ops.append(dist.P2POp(dist.irecv, buf, _global_rank(group, p[1]), group))
                    jobs.append((f, buf, p[2]))
                else:
                    nrows = cur[f] if prec == _lib.PREC_BF16 else ns[f]
                    ops.append(dist.P2POp(dist.isend, R[:nrows], _global_rank(group, p[1]), group))
            if ops:
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
            if jobs:
                merge_many([(items[f][0], cur[f], buf, rb, items[f][3]) for f, buf, rb in jobs])
                for f, _, rb in jobs:
                    cur[f] = min(ns[f], cur[f] + rb)
        s *= 2
    return results


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
    * At a refresh every layer's running factors are reduced across ranks to the
      layer's owner by the R-tree (:func:`rtree_reduce_many`: the merge order of
      ``ifkfac/triangular.py:207-220`` over ranks relabelled from the owner; the
      exchanges of all factors of a round batched in buckets of ``bucket_bytes``,
      their merges in batched folds), and the owner finalizes them (the row counts
      of all ranks scale them).  Other ranks keep no factors of that layer: it is
      solved on its owner only.
    * Gradients of the preconditioned layers are averaged across ranks (one
      ``all_reduce`` of a flat buffer) unless ``average_gradients=False`` (the
      caller already averages, e.g. under DDP).
    * The back-propagated rows δ a rank's hooks capture are those of that rank's
      loss.  With the usual loss, a mean over the rank's shard of a batch split in
      equal shards, each row is ``world`` times the row of the full-batch mean, so
      the merged R_G is scaled by ``delta_scale`` (default 1 / world; pass 1.0
      when each rank's loss is already normalised by the global batch).
    * Layer l's natural gradient and update run on rank ``l mod world`` only (its
      momentum buffer lives there); each owner then broadcasts the parameters of
      all its layers to the other ranks in one flat buffer (one broadcast per
      rank and step, not one per parameter).
    * If a collective of the refresh fails (a rank never posts its factor and the
      process group's timeout runs out), the factor update is skipped with a
      warning and the previous factors stay in use, the reference's handling of a
      refresh that cannot be computed (``ifkfac/ifkfac.py:207-223``); the running
      factors are cleared, since some may already hold a merged state.

    Construct it on every rank with the same model and arguments; ``step()`` is a
    collective."""

    def __init__(self, model, *args, group: Optional[dist.ProcessGroup] = None,
                 average_gradients: bool = True, delta_scale: Optional[float] = None,
                 bucket_bytes: int = 1 << 30, **kwargs):
        from .ifkfac import IFKFAC
        self.opt = IFKFAC(model, *args, **kwargs)
        self.group = group
        self.bucket_bytes = int(bucket_bytes)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.average_gradients = average_gradients
        self.delta_scale = 1.0 / self.world if delta_scale is None else float(delta_scale)
        self.owner = {m: i % self.world for i, m in enumerate(self.opt.hooks.linear_layers)}

    def __getattr__(self, name):
        return getattr(self.opt, name)

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.opt.zero_grad(set_to_none=set_to_none)

    def _merge_factors(self) -> bool:
        """R-tree merge of every factor; False (after a warning) when a collective failed."""
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
        entries = []  # (layer, 0 for X / 1 for delta, factor, row-count table)
        for li, m in enumerate(layers):
            for ti, (table, nrows) in enumerate(((h._fx, h._n_rows_X), (h._fg, h._n_rows_G))):
                n = int(width[li][ti])
                if n == 0:
                    continue  # no rank saw rows for this factor
                f = table[m]
                if f is None:
                    f = table[m] = Factor(n, dev, h.precision)
                entries.append((m, ti, f, nrows))
        try:
            got = rtree_reduce_many([(f.R, f.rows_R, f.rows_seen, f.prec) for _, _, f, _ in entries],
                                    [self.owner[m] for m, _, _, _ in entries], self.group,
                                    bucket_bytes=self.bucket_bytes)
        except (RuntimeError, dist.DistError) as e:  # timeouts and lost peers surface as these
            logger.warning("IFKFAC: R-tree merge failed (%s); factor update skipped", e)
            return False
        for (m, ti, f, nrows), (rows, total) in zip(entries, got):
            if self.owner[m] != self.rank:
                # not this rank's layer: its factors are finalised by the owner only
                f.rows_seen = 0
                continue
            f.rows_R, f.rows_seen = rows, total
            nrows[m] = total
            if ti == 1 and self.delta_scale != 1.0:
                f.R.mul_(self.delta_scale)  # R^T R scales with the square of the rows
        return True

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
            refresh_or_skip(self._merge_factors, opt._update_factors, opt.hooks.clear)
        todo = []
        for m in layers:
            lr, wd, mom = opt._get_module_hp(m)
            if lr is not None and self.owner[m] == self.rank:
                todo.append((m, lr, wd, mom))
        nats = opt._batched_natgrads([m for m, _, _, _ in todo])
        for m, lr, wd, mom in todo:
            opt._apply_preconditioner(m, lr, wd, mom, nats.get(m))
        # the owners' updated parameters go to every rank: one flat buffer per owner
        for o in range(self.world):
            params = [p for m in layers if self.owner[m] == o for p in m.parameters()]
            broadcast_flat(params, _global_rank(self.group, o), o == self.rank, self.group)
        return loss


def refresh_or_skip(merge, update, clear) -> bool:
    """The refresh of :class:`DistributedIFKFAC`: ``merge()`` (the R-tree of every
    factor, False when a collective failed), then ``update()`` (finalize, finite
    check, cast).  On a failed merge the update is skipped and ``clear()`` drops the
    running factors, which may hold a partly merged state; the factors already in
    use stay (the reference skips a refresh it cannot compute,
    ``ifkfac/ifkfac.py:207-223``).  Returns whether the factors were updated."""
    if merge():
        update()
        return True
    clear()
    return False


def broadcast_flat(params: Sequence[torch.Tensor], src: int, is_src: bool,
                   group: Optional[dist.ProcessGroup] = None) -> None:
    """Broadcast a list of tensors from global rank ``src`` as one flat buffer per
    dtype (one collective each instead of one per tensor); the receivers copy their
    slices back."""
    by_dtype = {}
    for p in params:
        by_dtype.setdefault(p.dtype, []).append(p)
    for dt, ps in by_dtype.items():
        if is_src:
            flat = torch.cat([p.data.reshape(-1) for p in ps])
        else:
            flat = torch.empty(sum(p.numel() for p in ps), dtype=dt, device=ps[0].device)
        dist.broadcast(flat, src=src, group=group)
        if not is_src:
            off = 0
            for p in ps:
                k = p.numel()
                p.data.copy_(flat[off:off + k].view_as(p.data))
                off += k
