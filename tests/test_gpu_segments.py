"""Segmented folds (ifk_tsqr_fold_segments): row tiles folded in one persistent
launch, in arrival order, give bit for bit the running factors of one
streaming fold per tile, because the reflector sequence (one sub-tile of rows
after another) is the same.  The damping rows appended in the same launch
(fused refresh) give the damped factor of the separate damping fold: bit for
bit when p is a power of 4 (the 1/sqrt(p) scaling is then exact), to rounding
otherwise."""
import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import ifk_oracle as ora
from ifkfac_b200 import _lib
from ifkfac_b200.engine import Factor, LayerCurvature, fold_batched, fold_segments

pytestmark = pytest.mark.gpu


def _inputs(rows, n, seed, dt):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = torch.exp(torch.rand(n, generator=g, device="cuda") * math.log(100.0))
    return (torch.randn(rows, n, generator=g, device="cuda") * s).to(dt)


def _truth(M, damping=None):
    R = ora.positive_diagonal_R(ora._qr_r(M.double().cpu().numpy()))
    if damping is None:
        return R
    n = M.shape[1]
    return ora.positive_diagonal_R(ora._qr_r(np.concatenate([R / math.sqrt(M.shape[0]),
                                                           math.sqrt(damping) * np.eye(n)], 0)))


def _rel(x, y):
    return float(np.linalg.norm(x - y) / np.linalg.norm(y))


@pytest.mark.parametrize("prec", [_lib.PREC_BF16, _lib.PREC_FP32])
@pytest.mark.parametrize("n,tiles", [(512, [512, 512, 200, 512, 300]), (320, [96, 96, 96, 96]),
                                     (1024, [768, 512, 256])])
def test_segments_bitwise_equal_per_tile_folds(prec, n, tiles):
    dt = torch.bfloat16 if prec == _lib.PREC_BF16 else torch.float32
    # tiles in separate allocations: the segments are not adjacent in memory
    xs = [_inputs(r, n, 10 + i, dt) for i, r in enumerate(tiles)]
    ds = [_inputs(r, n, 50 + i, dt) for i, r in enumerate(tiles)]
    a = (Factor(n, "cuda", prec), Factor(n, "cuda", prec))
    ws = None
    for x, d in zip(xs, ds):
        ws = fold_batched(a, (x, d), ws)
    b = (Factor(n, "cuda", prec), Factor(n, "cuda", prec))
    fold_segments(b, (xs, ds), None)
    torch.cuda.synchronize()
    for fa, fb in zip(a, b):
        assert fa.rows_R == fb.rows_R and fa.rows_seen == fb.rows_seen == sum(tiles)
        assert int(fb.status.item()) == 0
        assert torch.equal(fa.R, fb.R), float((fa.R - fb.R).abs().max())
    # and the factor is the QR of all rows
    rows = sum(tiles)
    if rows >= n:
        tol = 2e-2 if prec == _lib.PREC_BF16 else 1e-5
        assert _rel(b[0].R.double().cpu().numpy(), _truth(torch.cat(xs))) < tol


def test_segments_onto_running_factor():
    """Segments after earlier folds start from the running factor's rows."""
    n = 384
    xs = [_inputs(r, n, 90 + i, torch.bfloat16) for i, r in enumerate([200, 256, 512, 100])]
    a, b = Factor(n, "cuda", _lib.PREC_BF16), Factor(n, "cuda", _lib.PREC_BF16)
    for x in xs:
        a.fold(x)
    b.fold(xs[0])
    fold_segments((b,), (xs[1:],), None)
    torch.cuda.synchronize()
    assert torch.equal(a.R, b.R) and a.rows_R == b.rows_R == n


def test_segments_split_across_launches():
    """More segments than one launch holds (12), and more sub-tiles than one launch
    takes for n = 128 (384 waves: 384 sub-tiles), run as several launches."""
    n = 128
    tiles = [256] * 14 + [300]
    xs = [_inputs(r, n, 200 + i, torch.bfloat16) for i, r in enumerate(tiles)]
    a, b = Factor(n, "cuda", _lib.PREC_BF16), Factor(n, "cuda", _lib.PREC_BF16)
    for x in xs:
        a.fold(x)
    fold_segments((b,), (xs,), None)
    big = _inputs(384 * 256 + 700, n, 7, torch.bfloat16)
    c, d = Factor(n, "cuda", _lib.PREC_BF16), Factor(n, "cuda", _lib.PREC_BF16)
    c.fold(big[:1000])  # the sub-tiles restart at a segment boundary, as at a fold boundary
    c.fold(big[1000:])
    fold_segments((d,), ([big[:1000], big[1000:]],), None)
    torch.cuda.synchronize()
    assert torch.equal(a.R, b.R)
    assert torch.equal(c.R, d.R)
    assert _rel(d.R.double().cpu().numpy(), _truth(big)) < 5e-3


@pytest.mark.parametrize("rows,exact", [(4 * 256, True), (1000, False)])
def test_fused_refresh_matches_separate_damping_fold(rows, exact):
    n, tile = 256, 250
    X = _inputs(rows, n, 31, torch.bfloat16)
    D = _inputs(rows, n, 32, torch.bfloat16)
    out = []
    for consume in (False, True):
        lc = LayerCurvature(n, n, "cuda", _lib.PREC_BF16, torch.float32, tile, window=16)
        for lo in range(0, rows, tile):
            lc.fold(X[lo:lo + tile], D[lo:lo + tile])
        assert lc.refresh(1e-2, consume=consume)
        torch.cuda.synchronize()
        assert int(lc.status.item()) == 0
        assert lc.fx.consumed == consume
        out.append((lc.RX.clone(), lc.RG.clone()))
        if consume:
            with pytest.raises(RuntimeError):
                lc.fold(X[:tile], D[:tile])
            lc.clear()
            lc.fold(X[:tile], D[:tile])  # usable again after clear()
    for sep, fus, M in ((out[0][0], out[1][0], X), (out[0][1], out[1][1], D)):
        if exact:
            assert torch.equal(sep, fus), float((sep - fus).abs().max())
        else:
            assert _rel(fus.double().cpu().numpy(), sep.double().cpu().numpy()) < 1e-5
        t = _truth(M, 1e-2)
        assert _rel(fus.double().cpu().numpy(), t) < 2e-2


def test_fused_refresh_skips_trapezoidal_factor():
    """Too few rows for a square factor: nothing is consumed, refresh is skipped
    and the running factor keeps the rows (the reference's rank skip)."""
    n = 512
    lc = LayerCurvature(n, n, "cuda", _lib.PREC_BF16, torch.float32, 256, window=4)
    X = _inputs(300, n, 3, torch.bfloat16)
    lc.fold(X, X)
    assert not lc.refresh(1e-2, consume=True)
    assert not lc.fx.consumed and lc.fx.rows_R == 300 and lc.fx.rows_seen == 300


def test_segments_argument_errors():
    L = _lib.lib()
    n = 256
    R = torch.zeros(n, n, device="cuda")
    x = _inputs(300, n, 1, torch.bfloat16)
    ws = torch.empty(1 << 26, dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    a64 = lambda *v: (ctypes.c_int64 * len(v))(*v)

    def call(rows, ld, ptr, tail=None, rows_R=0, cols=n):
        seg = (_lib.Segment * 1)(_lib.Segment(ptr, ld, rows, None, 0, cols))
        return L.ifk_tsqr_fold_segments(
            1, (ctypes.c_void_p * 1)(R.data_ptr()), a64(n), a64(rows_R), a64(n), (ctypes.c_int * 1)(1), seg,
            _lib.BF16, (ctypes.c_double * 1)(tail) if tail is not None else None, _lib.PREC_BF16,
            st.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert call(-1, n, x.data_ptr()) == _lib.ERR_SHAPE
    assert call(300, n - 1, x.data_ptr()) == _lib.ERR_SHAPE
    assert call(300, n, None) == _lib.ERR_ARG
    assert call(300, n, x.data_ptr(), tail=float("nan")) == _lib.ERR_ARG
    assert call(300, n, x.data_ptr(), rows_R=n + 1) == _lib.ERR_SHAPE
    assert call(300, n, x.data_ptr(), cols=n - 2) == _lib.ERR_SHAPE
    assert call(0, n, None) == _lib.OK  # nothing to fold
    assert call(300, n, x.data_ptr()) == _lib.OK
    torch.cuda.synchronize()
    assert int(st.item()) == 0


def test_many_folds_share_launches_bitwise():
    """40 folds of mixed widths in one call (they share a launch: up to 64 folds and
    256 segments per launch) give every factor bit for bit as folding it alone."""
    from ifkfac_b200.engine import Factor, fold_segments
    g = torch.Generator(device="cuda").manual_seed(7)
    ns = [64 + 8 * (i % 33) for i in range(40)]
    chunks = [[torch.randn(300 + 37 * (i % 5), n, generator=g, device="cuda").bfloat16() for _ in range(1 + i % 3)]
              for i, n in enumerate(ns)]
    together = [Factor(n, "cuda", _lib.PREC_BF16) for n in ns]
    fold_segments(together, chunks, None)
    for n, cs, f in zip(ns, chunks, together):
        alone = Factor(n, "cuda", _lib.PREC_BF16)
        fold_segments([alone], [cs], None)
        torch.cuda.synchronize()
        assert int(f.status.item()) == 0
        assert torch.equal(f.R, alone.R)


@pytest.mark.parametrize("prec", [_lib.PREC_BF16, _lib.PREC_FP32])
def test_mixed_dtype_segments_in_one_call(prec):
    """fp32 and bf16 chunks in one call (each segment carries its type; an explicit
    precision): every factor as folding its chunks one call at a time."""
    from ifkfac_b200.engine import Factor, fold_segments
    g = torch.Generator(device="cuda").manual_seed(9)
    mk = lambda r, n, dt: torch.randn(r, n, generator=g, device="cuda").to(dt)
    lists = [[mk(300, 96, torch.float32), mk(200, 96, torch.float32)],
             [mk(500, 160, torch.bfloat16)],
             [mk(260, 128, torch.float32), mk(300, 128, torch.bfloat16), mk(90, 128, torch.float32)]]
    together = [Factor(c[0].shape[1], "cuda", prec) for c in lists]
    fold_segments(together, lists, None)
    for cs, f in zip(lists, together):
        alone = Factor(cs[0].shape[1], "cuda", prec)
        for c in cs:
            fold_segments([alone], [[c]], None)
        torch.cuda.synchronize()
        assert int(f.status.item()) == 0
        assert torch.equal(f.R, alone.R)
    with pytest.raises(TypeError):
        fold_segments([Factor(96, "cuda")], [[mk(10, 96, torch.float32), mk(10, 96, torch.bfloat16)]], None)


def test_fp32_segments_share_one_schedule_bitwise():
    """fp32 mode, segments of whole sub-tiles (the last one ragged) with damping
    rows: the segments of both folds run one wave schedule together, then the
    identity tails; every factor bit for bit as one fold per tile and then the
    damping rows as a trapezoidal chunk."""
    n, tiles, tail = 384, [512, 256, 768, 300], 0.7
    xs = [_inputs(r, n, 70 + i, torch.float32) for i, r in enumerate(tiles)]
    ds = [_inputs(r, n, 90 + i, torch.float32) for i, r in enumerate(tiles)]
    a = (Factor(n, "cuda", _lib.PREC_FP32), Factor(n, "cuda", _lib.PREC_FP32))
    ws = None
    for x, d in zip(xs, ds):
        ws = fold_batched(a, (x, d), ws)
    eye = torch.eye(n, device="cuda") * tail
    fold_batched(a, (eye, eye), ws, trapezoidal=True)
    b = (Factor(n, "cuda", _lib.PREC_FP32), Factor(n, "cuda", _lib.PREC_FP32))
    fold_segments(b, (xs, ds), None, ident_tail=[tail, tail])
    torch.cuda.synchronize()
    for fa, fb in zip(a, b):
        assert int(fb.status.item()) == 0
        assert torch.equal(fa.R, fb.R), float((fa.R - fb.R).abs().max())
