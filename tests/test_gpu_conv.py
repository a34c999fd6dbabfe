"""Conv2d inputs folded through in-place im2col (next-row f1).

The reference unfolds a Conv2d input with F.unfold into a (B * L, C * kh * kw)
matrix, optionally keeps a random subsample of its rows, and folds that
(ifkfac/activation_hooks.py:489-499, 522-530).  Here the fold's leaf loads read
each element from the NCHW image instead (Rows.conv2d, an ifk_segment with an
ifk_conv2d geometry).  The rows are the same values in the same order, so the
factor must equal, bit for bit, the fold of the materialised F.unfold rows, in
both precision modes, with padding, stride, dilation, rectangular kernels, a row
subsample, and a fold taller than one launch piece."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from ifkfac_b200 import _lib
from ifkfac_b200.engine import Factor, Rows, fold_segments

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _fold(n, segs, prec):
    f = Factor(n, DEV, prec)
    fold_segments([f], [segs], None)
    torch.cuda.synchronize()
    assert int(f.status.item()) == 0
    return f.R.clone(), f.rows_R


CASES = [
    dict(cin=3, cout=8, k=3, stride=1, padding=1, dilation=1, hw=(12, 12), B=4),
    dict(cin=5, cout=4, k=(3, 2), stride=(2, 1), padding=(1, 0), dilation=1, hw=(11, 9), B=3),
    dict(cin=16, cout=4, k=3, stride=2, padding=2, dilation=2, hw=(17, 13), B=2),
    dict(cin=64, cout=4, k=1, stride=1, padding=0, dilation=1, hw=(8, 8), B=2),
]


@pytest.mark.parametrize("prec", [_lib.PREC_BF16, _lib.PREC_FP32])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("subsample", [None, 150])
def test_conv_rows_fold_equals_unfold_rows(prec, dtype, case, subsample):
    c = CASES[case]
    g = torch.Generator(device=DEV).manual_seed(case)
    conv = nn.Conv2d(c["cin"], c["cout"], c["k"], stride=c["stride"], padding=c["padding"],
                     dilation=c["dilation"]).to(DEV)
    x = (torch.randn(c["B"], c["cin"], *c["hw"], device=DEV, generator=g) * 3).to(dtype)
    rows = Rows.conv2d(x, conv)
    idx = None
    if subsample is not None and rows.rows > subsample:
        idx = torch.randperm(rows.rows, device=DEV, generator=g)[:subsample]
        rows = Rows.conv2d(x, conv, idx)
    dense = rows.materialize()
    n = rows.cols
    assert dense.shape == (rows.rows, n)
    # the reference's own im2col of the same input, row for row
    ref = torch.nn.functional.unfold(x.float(), kernel_size=conv.kernel_size, dilation=conv.dilation,
                                     padding=conv.padding, stride=conv.stride)
    ref = ref.permute(0, 2, 1).reshape(-1, n)
    ref = ref[idx] if idx is not None else ref
    assert torch.equal(dense.float(), ref)
    R_img, r1 = _fold(n, [rows], prec)
    R_mat, r2 = _fold(n, [dense], prec)
    assert r1 == r2
    assert torch.equal(R_img, R_mat)


def test_conv_fold_taller_than_one_launch_piece():
    """131072 image rows at n = 27 (one launch piece holds 384 sub-tiles of 256 rows):
    the later pieces start further down the image, by row number."""
    g = torch.Generator(device=DEV).manual_seed(7)
    conv = nn.Conv2d(3, 4, 3, padding=1).to(DEV)
    x = torch.randn(32, 3, 64, 64, device=DEV, generator=g).to(torch.bfloat16)
    rows = Rows.conv2d(x, conv)
    assert rows.rows == 131072 and rows.cols == 27
    R_img, _ = _fold(27, [rows], _lib.PREC_BF16)
    R_mat, _ = _fold(27, [rows.materialize()], _lib.PREC_BF16)
    assert torch.equal(R_img, R_mat)
    # and the factor is that of all rows (the QR of the im2col matrix)
    A = rows.materialize().double().cpu().numpy()
    Rd = R_img.double().cpu().numpy()
    e = np.linalg.norm(Rd.T @ Rd - A.T @ A) / np.linalg.norm(A.T @ A)
    assert e < 1e-2, e


def test_ifkfac_on_a_conv_net_uses_image_rows():
    """The optimizer's hooks fold a Conv2d layer's input through the image rows; its
    factor equals the fold of the reference's unfolded rows."""
    from ifkfac_b200.ifkfac import IFKFAC
    torch.manual_seed(0)
    model = nn.Sequential(nn.Conv2d(3, 6, 3, padding=1), nn.ReLU(), nn.Flatten(), nn.Linear(6 * 64, 10)).to(DEV)
    opt = IFKFAC(model, lr=1e-2, damping=1e-2, factor_update_freq=1, max_conv_rows=0)
    x = torch.randn(16, 3, 8, 8, device=DEV)
    y = torch.randint(0, 10, (16,), device=DEV)
    loss = nn.functional.cross_entropy(model(x), y)
    loss.backward()
    conv = model[0]
    h = opt.hooks
    h.flush()
    torch.cuda.synchronize()
    fx = h._fx[conv]
    assert fx is not None and fx.n == 27
    R_hook = fx.R.clone()
    R_ref, _ = _fold(27, [Rows.conv2d(x, conv).materialize()], fx.prec)
    assert torch.equal(R_hook, R_ref)
