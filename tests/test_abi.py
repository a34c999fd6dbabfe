"""The C-ABI library loads on CPU-only hosts and exports every symbol include/ifk.h declares.

No compute call is made here (no GPU in this process); host-side queries that
touch no device (workspace sizes, status strings, argument validation that
fails before any CUDA call) are exercised.
"""
import ctypes

import pytest

from ifkfac_b200 import _lib


def test_library_exports_header_symbols():
    L = _lib.lib()
    names = _lib.header_symbols()
    assert len(names) >= 13
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_status_strings_and_version():
    assert b"sm_100a" in _lib.lib().ifk_version()
    for s in range(11):
        assert _lib.status_string(s)
    assert "rank" in _lib.status_string(_lib.ERR_RANK)


def test_workspace_sizes_are_host_only():
    L = _lib.lib()
    a = L.ifk_tsqr_fold_workspace(2048, 4096)
    assert a >= 2048 * 4096 * 4          # fp32 working copy of the chunk
    assert L.ifk_tsqr_fold_workspace(0, 0) == 0
    assert L.ifk_finalize_workspace(4096) >= 2 * 4096 * 4096 * 4
    assert L.ifk_update_workspace(10) >= 8


def test_argument_errors_before_any_gpu_work():
    L = _lib.lib()
    # rank-deficient factor: the reference skips it; the ABI says so without touching the device
    fake = ctypes.c_void_p(256)
    rc = L.ifk_finalize(fake, 64, 32, 64, 100.0, 1e-2, fake, 64, _lib.F32, 0, None, fake, 1 << 20, None)
    assert rc == _lib.ERR_RANK
    assert L.ifk_tsqr_fold(None, 64, 0, fake, 64, 10, 64, _lib.F32, 0, 0, None, fake, 1 << 20, None) == _lib.ERR_ARG
    assert L.ifk_tsqr_fold(fake, 32, 0, fake, 64, 10, 64, _lib.F32, 0, 0, None, fake, 1 << 20, None) == _lib.ERR_SHAPE
    assert L.ifk_tsqr_fold(fake, 64, 0, fake, 64, 10, 64, 7, 0, 0, None, fake, 1 << 20, None) == _lib.ERR_DTYPE
    assert L.ifk_tsqr_fold(fake, 64, 0, fake, 64, 10, 64, _lib.F32, 0, 0, None, fake, 16, None) == _lib.ERR_WORKSPACE
    assert L.ifk_natgrad(fake, 8, fake, 8, fake, 4, 9, fake, 8, 4, 8, 0, None, fake, 256, None) == _lib.ERR_DTYPE
    assert L.ifk_update(None, None, fake, 4, 0.1, 0.0, 0.0, 0.0, 0, None, 0, None) == _lib.ERR_ARG


def test_segment_struct_matches_header():
    """ctypes mirror of ifk_segment: the field order and offsets of include/ifk.h."""
    import re
    body = re.search(r"typedef struct ifk_segment \{(.*?)\} ifk_segment;", open(_lib.HEADER).read(), re.S).group(1)
    fields = re.findall(r"(\w+);", re.sub(r"/\*.*?\*/", "", body, flags=re.S))
    assert fields == [f for f, _ in _lib.Segment._fields_]
    assert ctypes.sizeof(_lib.Segment) == 64
    assert _lib.Segment.cols.offset == 40 and _lib.Segment.dtype.offset == 48 and _lib.Segment.conv.offset == 56
    body = re.search(r"struct ifk_conv2d \{(.*?)\};", open(_lib.HEADER).read(), re.S).group(1)
    names = [n for grp in re.findall(r"int\d+_t ([\w, ]+);", body) for n in grp.replace(" ", "").split(",")]
    assert names == [f for f, _ in _lib.Conv2d._fields_]
    assert ctypes.sizeof(_lib.Conv2d) == 64


def test_conv_segment_geometry_errors_before_any_gpu_work():
    """im2col segments: the columns must be C kh kw and the source rows N Ho Wo."""
    L = _lib.lib()
    a64 = lambda *v: (ctypes.c_int64 * len(v))(*v)
    geo = _lib.Conv2d(2, 3, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1)  # Ho = Wo = 8
    n = 27

    def call(cols=27, src=2 * 64, rows=100, g=geo):
        segs = (_lib.Segment * 1)(_lib.Segment(0x1000, 0, rows, None, src, cols, 0, 0, ctypes.pointer(g)))
        return L.ifk_tsqr_fold_segments(1, (ctypes.c_void_p * 1)(0x2000), a64(n), a64(0), a64(n),
                                        (ctypes.c_int * 1)(1), segs, _lib.BF16, None, _lib.PREC_BF16, None,
                                        None, 0, None)
    assert call() == _lib.ERR_WORKSPACE  # valid geometry: only the missing workspace is refused
    assert call(cols=26) == _lib.ERR_SHAPE
    assert call(src=2 * 63) == _lib.ERR_SHAPE
    assert call(rows=2 * 64 + 1) == _lib.ERR_SHAPE  # more rows than the image has
    assert call(g=_lib.Conv2d(2, 3, 8, 8, 3, 3, 0, 1, 1, 1, 1, 1)) == _lib.ERR_SHAPE  # zero stride


def test_segment_fold_argument_errors_before_any_gpu_work():
    L = _lib.lib()
    a64 = lambda *v: (ctypes.c_int64 * len(v))(*v)
    n = 64
    seg = lambda rows=100, ld=64, cols=64, chunk=0x1000, idx=None, src=0, dt=0: (_lib.Segment * 1)(
        _lib.Segment(chunk, ld, rows, idx, src, cols, dt, 0))
    call = lambda segs, ntail=None, rows_R=0, cdt=_lib.BF16, prec=_lib.PREC_BF16: L.ifk_tsqr_fold_segments(
        1, (ctypes.c_void_p * 1)(0x2000), a64(n), a64(rows_R), a64(n), (ctypes.c_int * 1)(1), segs, cdt,
        (ctypes.c_double * 1)(ntail) if ntail is not None else None, prec, None, None, 0, None)
    assert call(seg(cols=62)) == _lib.ERR_SHAPE            # neither n nor n - 1 columns
    assert call(seg(cols=63, ld=62)) == _lib.ERR_SHAPE     # leading dimension below the columns
    assert call(seg(rows=-1)) == _lib.ERR_SHAPE
    assert call(seg(chunk=None)) == _lib.ERR_ARG
    assert call(seg(idx=0x3000, src=0)) == _lib.ERR_SHAPE  # gathered rows need the source's row count
    assert call(seg(), ntail=float("nan")) == _lib.ERR_ARG
    assert call(seg(), rows_R=n + 1) == _lib.ERR_SHAPE
    assert call(seg(rows=0)) == _lib.OK                    # nothing to fold
    assert call(seg(cols=63)) == _lib.ERR_WORKSPACE        # valid (bias column), but no workspace
    per = _lib.PER_SEGMENT_DTYPE
    assert call(seg(dt=_lib.BF16), cdt=per) == _lib.ERR_WORKSPACE          # per-segment dtype, valid
    assert call(seg(dt=5), cdt=per) == _lib.ERR_DTYPE                      # a segment's dtype is checked
    assert call(seg(dt=_lib.F32), cdt=per, prec=_lib.PREC_AUTO) == _lib.ERR_ARG  # needs an explicit precision
    ws = L.ifk_tsqr_fold_segments_workspace(1, a64(n), (ctypes.c_int * 1)(1), seg(rows=1000), None)
    assert ws >= L.ifk_tsqr_fold_workspace(1000, n) // 2 and ws > 0
    wt = L.ifk_tsqr_fold_segments_workspace(1, a64(n), (ctypes.c_int * 1)(1), seg(rows=1000),
                                            (ctypes.c_double * 1)(1.0))
    assert wt >= ws                                       # the damping rows add sub-tiles


def test_fold_workspace_stops_at_one_launch_piece():
    """A fold taller than one persistent launch runs as several launches over one
    workspace, so its workspace stops growing at the piece size: 384 - 2 (CB - 1)
    sub-tiles of 256 rows, 322 at n = 4096 (CB = 32 column blocks).  Chunks of
    2048 rows keep the fp32 path's share fixed."""
    L = _lib.lib()
    n = 4096
    a64 = lambda *v: (ctypes.c_int64 * len(v))(*v)

    def ws(nchunks):
        segs = (_lib.Segment * nchunks)(*[_lib.Segment(0x1000, n, 2048, None, 0, n, 0, 0)
                                          for _ in range(nchunks)])
        return L.ifk_tsqr_fold_segments_workspace(1, a64(n), (ctypes.c_int * 1)(nchunks), segs, None)

    piece = 322 // 8  # whole chunks of 8 sub-tiles below the piece size
    assert ws(piece) < ws(piece + 1) == ws(piece + 2) == ws(200)
    assert ws(1) < ws(2) < ws(piece)


def test_fp32_segments_workspace_covers_the_concatenation():
    """ifk_tsqr_fold_segments_fp32_workspace: at least the segments workspace, and
    an fp32 copy of all of a fold's rows (so it grows with the number of chunks,
    where the segments workspace stops at one launch piece); the damping rows need
    n rows of it."""
    L = _lib.lib()
    n = 1024
    a64 = lambda *v: (ctypes.c_int64 * len(v))(*v)

    def both(nchunks, rows=512, tail=None):
        segs = (_lib.Segment * nchunks)(*[_lib.Segment(0x1000, n, rows, None, 0, n, 0, 0)
                                          for _ in range(nchunks)])
        t = (ctypes.c_double * 1)(tail) if tail else None
        args = (1, a64(n), (ctypes.c_int * 1)(nchunks), segs, t)
        return L.ifk_tsqr_fold_segments_workspace(*args), L.ifk_tsqr_fold_segments_fp32_workspace(*args)

    for k in (1, 4, 40, 400):
        base, cat = both(k)
        assert cat >= base > 0
        assert cat >= k * 512 * n * 4  # every row of the fold, fp32
    assert both(400)[1] > both(40)[1] > both(4)[1]
    assert both(1, rows=64, tail=1.0)[1] >= n * n * 4  # the identity tail takes n rows
    assert L.ifk_tsqr_fold_segments_fp32_workspace(0, None, None, None, None) == 0
