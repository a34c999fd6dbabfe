"""ifk_natgrad_update: the natural gradient and the momentum / lr update in one
call (apply_vered, ifkfac/triangular.py:551-656, then the per-layer epilogue of
ifkfac/ifkfac.py:394-413).  The result must be that of ifk_natgrad followed by
ifk_update, bit for bit, on every path."""
import ctypes
import math

import numpy as np
import pytest

from ifkfac_b200 import _lib
from oracle import ifk_oracle as O

pytestmark = pytest.mark.gpu


def _factor(rng, p, n, lam=1e-2):
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    X = O.bf16_round((rng.standard_normal((p, n)) * s).astype(np.float32))
    return O.get_factor(O.streaming_tsqr_update(None, X), p, lam)


@pytest.mark.parametrize("n_out,n_in,prec,rdt", [
    (384, 520, _lib.PREC_BF16, "bf16"),    # persistent solves
    (1024, 768, _lib.PREC_BF16, "bf16"),
    (100, 130, _lib.PREC_BF16, "bf16"),    # orders off the multiple of 8: solves, then the update pass
    (384, 520, _lib.PREC_FP32, "f32"),     # fp32 mode
])
def test_natgrad_update_matches_the_two_calls(n_out, n_in, prec, rdt):
    import torch
    L = _lib.lib()
    rng = np.random.default_rng(n_out + n_in + prec)
    dt = torch.bfloat16 if rdt == "bf16" else torch.float32
    code = _lib.BF16 if rdt == "bf16" else _lib.F32
    RX = torch.from_numpy(_factor(rng, 2 * n_in, n_in)).cuda().to(dt)
    RG = torch.from_numpy(_factor(rng, 2 * n_out, n_out)).cuda().to(dt)
    stream = torch.cuda.current_stream().cuda_stream
    lr, mom, wd = 1e-3, 0.9, 1e-2
    W0 = torch.from_numpy((rng.standard_normal((n_out, n_in)) * 1e-2).astype(np.float32)).cuda()
    Wa, Wb = W0.clone(), W0.clone()
    ba, bb = torch.empty_like(W0), torch.empty_like(W0)
    ws_n = torch.empty(L.ifk_natgrad_workspace(n_out, n_in), dtype=torch.uint8, device="cuda")
    ws_u = torch.empty(L.ifk_natgrad_update_workspace(n_out, n_in), dtype=torch.uint8, device="cuda")
    ws_up = torch.empty(L.ifk_update_workspace(n_out * n_in), dtype=torch.uint8, device="cuda")
    nat = torch.empty_like(W0)
    for step in range(2):
        g = torch.from_numpy((rng.standard_normal((n_out, n_in)) * 1e-2).astype(np.float32)).cuda()
        g_keep = g.clone()
        new = 1 if step == 0 else 0
        _lib.check(L.ifk_natgrad(g.data_ptr(), n_in, RX.data_ptr(), n_in, RG.data_ptr(), n_out, code,
                                 nat.data_ptr(), n_in, n_out, n_in, prec, None, ws_n.data_ptr(), ws_n.numel(),
                                 stream), "ifk_natgrad")
        _lib.check(L.ifk_update(Wa.data_ptr(), ba.data_ptr(), nat.data_ptr(), n_out * n_in, lr, mom, wd, 0.0, new,
                                ws_up.data_ptr(), ws_up.numel(), stream), "ifk_update")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.check(L.ifk_natgrad_update(g.data_ptr(), n_in, RX.data_ptr(), n_in, RG.data_ptr(), n_out, code,
                                        Wb.data_ptr(), bb.data_ptr(), n_out, n_in, lr, mom, wd, new, prec,
                                        st.data_ptr(), ws_u.data_ptr(), ws_u.numel(), stream),
                   "ifk_natgrad_update")
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert torch.equal(g, g_keep)  # the gradient is not modified
        # buf first: on the first step it is the natural gradient itself
        assert torch.equal(ba, bb), (step, float((ba - bb).abs().max()), float(ba.abs().max()))
        assert torch.equal(Wa, Wb), (step, float((Wa - Wb).abs().max()))
