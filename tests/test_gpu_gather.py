"""Rows read in place by the fold (ifk_segment row_index / cols): a random row
subsample and an appended column of ones, as the reference's hooks build them
(ifkfac/activation_hooks.py:531-543), give bit for bit the factor of the
materialised rows, in both precision modes."""
import math

import numpy as np
import pytest
import torch

from ifkfac_b200 import _lib
from ifkfac_b200.engine import Factor, Rows, fold_segments

pytestmark = pytest.mark.gpu


def _data(rows, cols, seed, dt):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = torch.exp(torch.rand(cols, generator=g, device="cuda") * math.log(100.0))
    return (torch.randn(rows, cols, generator=g, device="cuda") * s).to(dt)


@pytest.mark.parametrize("prec,dt", [(_lib.PREC_BF16, torch.bfloat16), (_lib.PREC_FP32, torch.float32)])
@pytest.mark.parametrize("cols,src,take,ones", [(127, 900, 700, True), (256, 600, 600, False),
                                                (255, 1000, 333, True), (64, 5000, 2048, True)])
def test_gathered_rows_equal_materialised(prec, dt, cols, src, take, ones):
    x = _data(src, cols, 5 + cols, dt)
    g = torch.Generator(device="cuda").manual_seed(cols)
    idx = torch.randperm(src, device="cuda", generator=g)[:take]
    r = Rows(x, idx, ones)
    n = r.cols
    a, b = Factor(n, "cuda", prec), Factor(n, "cuda", prec)
    fold_segments((a,), ([r],), None)
    fold_segments((b,), ([r.materialize()],), None)
    torch.cuda.synchronize()
    assert int(a.status.item()) == 0
    assert a.rows_R == b.rows_R == min(n, take)
    assert torch.equal(a.R, b.R), float((a.R - b.R).abs().max())


def test_gathered_rows_over_several_launches():
    """A gathered segment longer than one launch takes continues with the rest of
    its index array in the next launch."""
    n = 128
    x = _data(400 * 256, n - 1, 11, torch.bfloat16)
    idx = torch.randperm(x.shape[0], device="cuda")[: 390 * 256 + 77]
    r = Rows(x, idx, ones=True)
    a, b = Factor(n, "cuda", _lib.PREC_BF16), Factor(n, "cuda", _lib.PREC_BF16)
    fold_segments((a,), ([r],), None)
    fold_segments((b,), ([r.materialize()],), None)
    torch.cuda.synchronize()
    assert torch.equal(a.R, b.R)


def test_several_gathered_segments_and_plain_chunks():
    n = 200
    xs = [_data(300 + 50 * i, n, 30 + i, torch.bfloat16) for i in range(3)]
    segs = [Rows(xs[0], torch.arange(299, -1, -2, device="cuda")), xs[1],
            Rows(xs[2], torch.randperm(400, device="cuda")[:250])]
    a, b = Factor(n, "cuda", _lib.PREC_BF16), Factor(n, "cuda", _lib.PREC_BF16)
    fold_segments((a,), (segs,), None)
    for c in segs:
        fold_segments((b,), ([c],), None)
    torch.cuda.synchronize()
    assert torch.equal(a.R, b.R)
    mat = torch.cat([s.materialize() if isinstance(s, Rows) else s for s in segs], 0)
    c = Factor(n, "cuda", _lib.PREC_BF16)
    fold_segments((c,), ([Rows(mat)],), None)
    torch.cuda.synchronize()
    # one chunk of all rows: other sub-tile boundaries, same factor to rounding
    rel = float((c.R - a.R).norm() / a.R.norm())
    assert rel < 2e-2


def test_out_of_range_index_is_reported():
    n = 96
    x = _data(200, n, 3, torch.bfloat16)
    idx = torch.arange(150, device="cuda")
    idx[7] = 200  # one past the end
    f = Factor(n, "cuda", _lib.PREC_BF16)
    fold_segments((f,), ([Rows(x, idx)],), None)
    torch.cuda.synchronize()
    assert int(f.status.item()) == _lib.ERR_ARG
    g = Factor(n, "cuda", _lib.PREC_FP32)
    fold_segments((g,), ([Rows(x.float(), idx)],), None)
    torch.cuda.synchronize()
    assert int(g.status.item()) == _lib.ERR_ARG


@pytest.mark.parametrize("autocast", [False, True])
def test_hooks_read_subsample_and_bias_in_place(autocast):
    """The hooks' in-place rows give the factors of the materialised rows (an
    identity chunk transform forces the copies), in streaming and deferred mode."""
    from ifkfac_b200.activation_hooks import RawActivationHooks
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(48, 64), torch.nn.ReLU(), torch.nn.Linear(64, 40)).cuda()
    x = torch.randn(8, 300, 48, device="cuda")
    out = {}
    for key in ("rows", "copies", "deferred"):
        hooks = RawActivationHooks(model, damping=1e-2, augment_bias=True, max_seq_rows=1000,
                                   deferred=key == "deferred", deferred_window=2)
        if key == "copies":
            hooks.chunk_transform_X = lambda c: c
            hooks.chunk_transform_G = lambda c: c
        hooks.enable()
        for it in range(3):
            torch.manual_seed(100 + it)  # the same row subsample in every run
            model.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
                y = model(x * (1 + it))
            y.float().square().mean().backward()
        out[key] = {m: (rx.clone(), rg.clone()) for m, (rx, rg) in hooks.get_factors().items()}
        hooks.remove()
    assert len(out["rows"]) == 2
    for m in out["rows"]:
        for a, b, c in zip(out["rows"][m], out["copies"][m], out["deferred"][m]):
            assert torch.isfinite(a).all()
            # same rows, same sub-tiles (segments restart at chunk boundaries): same bits
            assert torch.equal(a, b), float((a - b).abs().max())
            assert torch.equal(a, c), float((a - c).abs().max())
