"""Batch-sharded TSQR: gather of the local factors and the reference ``tsqr``
merge tree (``ifkfac/triangular.py:207-220``).

CPU tests run world_size 2 and 3 ranks on gloo with the oracle's merge injected
(the oracle is the checker; the library's merge is the GPU fold).  The GPU
test runs the library's merge on factors held by one device."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import ifk_oracle as ora
from ifkfac_b200 import distributed as D

N = 24


def _rows_for(rank):
    # rank 1 holds fewer rows than columns (trapezoid), rank 2 (if any) none
    return {0: 40, 1: 13, 2: 0, 3: 30, 4: 7}[rank]


def _data(rank):
    rng = np.random.default_rng(100 + rank)
    s = np.exp(rng.uniform(0, np.log(100.0), N))
    return rng.standard_normal((_rows_for(rank), N)) * s


def _local_factor(X):
    R = np.zeros((N, N))
    if X.shape[0]:
        r = ora.positive_diagonal_R(ora._qr_r(X))
        R[: r.shape[0]] = r
    return R


def _oracle_merge(Ra, ra, Rb, rb):
    """[Ra[:ra]; Rb[:rb]] -> Ra (positive diagonal, missing rows zero), as the GPU fold."""
    k = min(rb, N)
    if k == 0:
        return ra
    stacked = np.concatenate([Ra[:ra].numpy(), Rb[:k].numpy()], 0)
    r = ora.positive_diagonal_R(ora._qr_r(stacked))
    Ra.zero_()
    Ra[: r.shape[0]] = torch.from_numpy(r)
    return min(N, ra + k)


def _worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        X = _data(rank)
        R = torch.from_numpy(_local_factor(X))
        rows, seen = D.rtree_merge(R, min(N, X.shape[0]), X.shape[0], merge=_oracle_merge)
        np.save(os.path.join(outdir, f"r{rank}.npy"), R.numpy())
        np.save(os.path.join(outdir, f"c{rank}.npy"), np.array([rows, seen]))
    finally:
        torch.distributed.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3, 5])
def test_rtree_merge_gloo_matches_tsqr(tmp_path, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    Rs = [np.load(tmp_path / f"r{r}.npy") for r in range(world)]
    cs = [np.load(tmp_path / f"c{r}.npy") for r in range(world)]
    total = sum(_rows_for(r) for r in range(world))
    for r in range(world):
        np.testing.assert_array_equal(Rs[r], Rs[0])  # the same factor on every rank
        assert list(cs[r]) == [min(N, total), total]
    # the reference tree over the same local factors, and the plain QR of all rows
    allX = np.concatenate([_data(r) for r in range(world)], 0)
    ref = ora.positive_diagonal_R(ora._qr_r(allX))
    np.testing.assert_allclose(Rs[0][: ref.shape[0]], ref, rtol=0, atol=1e-9 * np.abs(ref).max())


def test_tree_merge_order_is_the_reference_tree():
    # records the merge order: pairs of adjacent entries, odd one carried forward
    log = []

    def merge(a, na, b, nb):
        log.append((int(a[0]), int(b[0])))
        return na + nb

    bufs = [torch.tensor([float(i)]) for i in range(5)]
    out, rows = D.tree_merge(bufs, [1] * 5, merge)
    assert log == [(0, 1), (2, 3), (0, 2), (0, 4)]
    assert rows == 5 and int(out[0]) == 0


def test_tree_merge_rejects_mismatched_counts():
    with pytest.raises(ValueError):
        D.tree_merge([torch.zeros(2, 2)], [1, 2])


@pytest.mark.gpu
def test_fold_merge_on_device_matches_oracle_tsqr():
    dev = torch.device("cuda")
    n, per = 96, [200, 60, 0, 150]
    rng = np.random.default_rng(7)
    s = np.exp(rng.uniform(0, np.log(100.0), n))
    blocks = [rng.standard_normal((p, n)) * s for p in per]
    factors, rows = [], []
    for X in blocks:
        R = np.zeros((n, n))
        if X.shape[0]:
            r = ora.positive_diagonal_R(ora._qr_r(X))
            R[: r.shape[0]] = r
        factors.append(torch.tensor(R, dtype=torch.float32, device=dev))
        rows.append(min(n, X.shape[0]))
    out, nrows = D.tree_merge(factors, rows)
    torch.cuda.synchronize()
    ref = ora.positive_diagonal_R(ora._qr_r(np.concatenate(blocks, 0)))
    err = np.linalg.norm(out.cpu().numpy().astype(np.float64) - ref) / np.linalg.norm(ref)
    assert nrows == n and err < 1e-5, err


def _factor_data(rank, f, n):
    rng = np.random.default_rng(1000 + 17 * f + rank)
    s = np.exp(rng.uniform(0, np.log(100.0), n))
    return rng.standard_normal(((_rows_for(rank) + 5 * f) % 45, n)) * s


def _oracle_merge_many(jobs):
    for Ra, ra, Rb, rb, _ in jobs:
        n = Ra.shape[1]
        k = min(rb, n)
        if k == 0:
            continue
        stacked = np.concatenate([Ra[:ra].numpy(), Rb[:k].numpy()], 0)
        r = ora.positive_diagonal_R(ora._qr_r(stacked))
        Ra.zero_()
        Ra[: r.shape[0]] = torch.from_numpy(r)


MANY_N = [24, 24, 10, 24, 16]


def _reduce_many_worker(rank, world, port, outdir, prec):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        items = []
        for f, n in enumerate(MANY_N):
            X = _factor_data(rank, f, n)
            R = np.zeros((n, n))
            if X.shape[0]:
                r = ora.positive_diagonal_R(ora._qr_r(X))
                R[: r.shape[0]] = r
            items.append((torch.from_numpy(R), min(n, X.shape[0]), X.shape[0], prec))
        owners = [f % world for f in range(len(MANY_N))]
        owners[-1] = world - 1
        # small buckets: the exchanges of a round go in several batches
        got = D.rtree_reduce_many(items, owners, merge_many=_oracle_merge_many, bucket_bytes=2 * 24 * 24 * 8)
        for f, (R, _, _, _) in enumerate(items):
            if owners[f] == rank:
                np.save(os.path.join(outdir, f"m{f}.npy"), R.numpy())
        np.save(os.path.join(outdir, f"g{rank}.npy"), np.array(got))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world,prec", [(2, 1), (3, 2), (5, 2)])
def test_rtree_reduce_many_gloo_reduces_every_factor_to_its_owner(tmp_path, world, prec):
    # prec 2 (bf16 mode) sends only the meaningful rows of a factor, 1 (fp32 mode) the whole factor
    mp.spawn(_reduce_many_worker, args=(world, _free_port(), str(tmp_path), prec), nprocs=world, join=True)
    gots = [np.load(tmp_path / f"g{r}.npy") for r in range(world)]
    for r in range(world):
        np.testing.assert_array_equal(gots[r], gots[0])  # the same counts on every rank
    for f, n in enumerate(MANY_N):
        allX = np.concatenate([_factor_data(r, f, n) for r in range(world)], 0)
        assert list(gots[0][f]) == [min(n, allX.shape[0]), allX.shape[0]]
        ref = ora.positive_diagonal_R(ora._qr_r(allX))
        got = np.load(tmp_path / f"m{f}.npy")
        np.testing.assert_allclose(got[: ref.shape[0]], ref, rtol=0, atol=1e-9 * np.abs(ref).max())


def _silent_rank_worker(rank, world, port, outdir):
    """Rank 1 never posts its factor (it does not enter the merge); the others must
    give up within the process group's timeout and keep their local factor."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=3))
    done = os.path.join(outdir, "done")
    if rank == 1:
        # stay alive, silent, until the others have finished (no collective at all)
        import time
        t0 = time.time()
        while len([f for f in os.listdir(outdir) if f.startswith("res")]) < world - 1 and time.time() - t0 < 60:
            time.sleep(0.1)
        open(done, "w").close()
        os._exit(0)
    X = _data(rank)
    R = torch.from_numpy(_local_factor(X))
    before = R.clone()
    import time
    t0 = time.time()
    got = D.merge_or_skip(R, min(N, X.shape[0]), X.shape[0], merge=_oracle_merge)
    dt = time.time() - t0
    np.save(os.path.join(outdir, f"res{rank}.npy"),
            np.array([got is None, bool(torch.equal(R, before)), dt]))
    import time as _t
    t1 = _t.time()
    while not os.path.exists(done) and _t.time() - t1 < 60:
        _t.sleep(0.1)
    os._exit(0)  # the group is broken: leave without a collective teardown


def test_rank_that_never_posts_its_factor_times_out_on_the_host(tmp_path):
    world = 3
    mp.spawn(_silent_rank_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in (0, 2):
        skipped, unchanged, secs = np.load(tmp_path / f"res{r}.npy")
        assert skipped and unchanged, r
        assert secs < 30, secs  # bounded by the 3 s timeout of each failing collective


def test_refresh_is_skipped_when_the_merge_fails():
    calls = []
    ok = D.refresh_or_skip(lambda: False, lambda: calls.append("update"), lambda: calls.append("clear"))
    assert not ok and calls == ["clear"]
    calls.clear()
    ok = D.refresh_or_skip(lambda: True, lambda: calls.append("update"), lambda: calls.append("clear"))
    assert ok and calls == ["update"]


def _bcast_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ps = [torch.full((3, 2), float(rank)), torch.full((5,), 10.0 + rank),
              torch.full((2,), 20 + rank, dtype=torch.int64)]
        D.broadcast_flat(ps, src=1, is_src=(rank == 1))
        np.save(os.path.join(outdir, f"b{rank}.npy"),
                np.concatenate([p.double().reshape(-1).numpy() for p in ps]))
    finally:
        torch.distributed.destroy_process_group()


def test_broadcast_flat_gloo(tmp_path):
    mp.spawn(_bcast_worker, args=(3, _free_port(), str(tmp_path)), nprocs=3, join=True)
    want = np.concatenate([np.full(6, 1.0), np.full(5, 11.0), np.full(2, 21.0)])
    for r in range(3):
        np.testing.assert_array_equal(np.load(tmp_path / f"b{r}.npy"), want)
