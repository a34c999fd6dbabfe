"""ifk_natgrad_noalloc: the workspace-free natural gradient, called through the C ABI.

This entry point exists for callers that cannot allocate device memory where
they need the natural gradient (for example a step run inside another
framework's operator, whose memory belongs to that framework's pool).  Its
scratch is a fixed array inside the library, so the test checks that two calls
in a row (the second sees the first call's leftovers in that array) both
match ifk_natgrad, which is given a caller-allocated workspace.

This file is collected last so that a run stopping at the first failure has
already run every other test; it passes alone in a fresh process as well.
"""
import ctypes
import math

import numpy as np
import pytest

from ifkfac_b200 import _lib
from oracle import ifk_oracle as O
from tests.golden_io import rel


def _factor(rng, p, n, lam=1e-2):
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    X = O.bf16_round((rng.standard_normal((p, n)) * s).astype(np.float32))
    return O.bf16_round(O.get_factor(O.streaming_tsqr_update(None, X), p, lam))


def test_noalloc_rejects_sizes_above_its_limit():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    n = _lib.NOALLOC_MAX_N + 1
    rc = L.ifk_natgrad_noalloc(fake, n, fake, n, fake, 8, _lib.BF16, fake, n, 8, n, _lib.PREC_BF16,
                               None, None)
    assert rc == _lib.ERR_LIMIT
    assert "no-allocation" in _lib.status_string(rc)


def _two_calls(n_out, n_in, prec, rng, tol_ref, tol_oracle):
    import torch
    L = _lib.lib()
    RX = torch.from_numpy(_factor(rng, 2 * n_in, n_in)).cuda().to(torch.bfloat16)
    RG = torch.from_numpy(_factor(rng, 2 * n_out, n_out)).cuda().to(torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        gW = torch.from_numpy((rng.standard_normal((n_out, n_in)) * 1e-2).astype(np.float32)).cuda()
        ref = torch.empty_like(gW)
        ws = torch.empty(L.ifk_natgrad_workspace(n_out, n_in), dtype=torch.uint8, device="cuda")
        _lib.check(L.ifk_natgrad(gW.data_ptr(), n_in, RX.data_ptr(), n_in, RG.data_ptr(), n_out,
                                 _lib.BF16, ref.data_ptr(), n_in, n_out, n_in, prec, None,
                                 ws.data_ptr(), ws.numel(), stream), "ifk_natgrad")
        out = torch.full_like(gW, float("nan"))
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.check(L.ifk_natgrad_noalloc(gW.data_ptr(), n_in, RX.data_ptr(), n_in, RG.data_ptr(),
                                         n_out, _lib.BF16, out.data_ptr(), n_in, n_out, n_in, prec,
                                         status.data_ptr(), stream), "ifk_natgrad_noalloc")
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        # ifk_natgrad runs the persistent solves where they apply, the no-allocation
        # entry point the per-block-row ones: same numerics, agreement to the
        # bf16-path tolerance of the other tests
        assert rel(out.cpu().numpy(), ref.cpu().numpy()) < tol_ref, call
        want = O.apply_vered(gW.cpu().numpy(), RX.float().cpu().numpy(), RG.float().cpu().numpy(),
                             r_is_bf16=True)
        assert rel(out.cpu().numpy(), want) < tol_oracle, call


@pytest.mark.gpu
def test_noalloc_bf16_matches_natgrad_on_two_calls():
    """bf16 mode: the solves use the fixed scratch array (diagonal-block inverses)."""
    _two_calls(384, 520, _lib.PREC_BF16, np.random.default_rng(2024 + _lib.PREC_BF16), 5e-3, 5e-3)


@pytest.mark.gpu
def test_noalloc_fp32_argument_path():
    """fp32 mode: the solves run on the CUDA cores and never touch the scratch array,
    so this case checks the argument path and the result only."""
    _two_calls(384, 520, _lib.PREC_FP32, np.random.default_rng(2024 + _lib.PREC_FP32), 5e-3, 1e-5)


@pytest.mark.gpu
def test_noalloc_bf16_at_its_size_limit():
    """The largest order the array serves (4096), next to an order that is not a
    multiple of the 128-row blocks, so the scratch is filled to its end."""
    n = _lib.NOALLOC_MAX_N
    _two_calls(n, n - 1, _lib.PREC_BF16, np.random.default_rng(77), 5e-3, 5e-3)
