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
    return {0: 40, 1: 13, 2: 0, 3: 30}[rank]


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


@pytest.mark.parametrize("world", [2, 3])
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
