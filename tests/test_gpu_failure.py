"""Failure detection on the device without a GPU fault.

Every cross-CTA wait of the persistent fold is bounded.  A wait that gives up
sets the launch's abort word (the other CTAs stop at their next poll), writes
IFK_ERR_TIMEOUT to the caller's status word and returns; the context stays
usable.  The test withholds a dependency from the host side
(IFK_FOLD_DEBUG_WITHHOLD: the first panel of the fold is never published, and
the waits give up after milliseconds), so the waits on it run out, then checks
the status word and that the next, normal fold on the same device is correct.
This is the device half of the reference's failure handling: a layer whose
curvature could not be computed is skipped (ifkfac/ifkfac.py:207-223) and its
raw gradient used (:482-489).
"""
import ctypes
import math

import numpy as np
import pytest

from ifkfac_b200 import _lib
from oracle import ifk_oracle as O
from tests.golden_io import rel


def test_withhold_flag_is_rejected_outside_the_persistent_fold():
    """Host-side validation: the debug flag only applies to the bf16 persistent fold,
    and an fp32-mode call with it is refused before anything is queued."""
    L = _lib.lib()
    n, rows = 64, 64
    fake = ctypes.c_void_p(256)
    ws = L.ifk_tsqr_fold_workspace(rows, n)
    rc = L.ifk_tsqr_fold(fake, n, 0, fake, n, rows, n, _lib.F32, _lib.PREC_FP32, _lib.FOLD_DEBUG_WITHHOLD,
                         None, fake, ws, None)
    assert rc == _lib.ERR_ARG
    rc = L.ifk_tsqr_fold(fake, n, 0, fake, n, rows, n, _lib.F32, _lib.PREC_FP32, 1 << 12, None, fake, ws, None)
    assert rc == _lib.ERR_ARG


@pytest.mark.gpu
def test_withheld_panel_times_out_and_the_device_stays_usable():
    import torch
    L = _lib.lib()
    rng = np.random.default_rng(5)
    n, rows = 256, 512
    s = np.exp(rng.uniform(0, math.log(100.0), n))
    X = O.bf16_round((rng.standard_normal((rows, n)) * s).astype(np.float32))
    x = torch.from_numpy(X).cuda().to(torch.bfloat16)
    ws = torch.empty(L.ifk_tsqr_fold_workspace(rows, n), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    R = torch.zeros(n, n, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.ifk_tsqr_fold(R.data_ptr(), n, 0, x.data_ptr(), n, rows, n, _lib.BF16, _lib.PREC_BF16,
                         _lib.FOLD_DEBUG_WITHHOLD, status.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    assert rc == _lib.OK  # queued; the failure is found on the device
    torch.cuda.synchronize()  # the kernel returned: every wait was bounded
    assert int(status.item()) == _lib.ERR_TIMEOUT
    # the context is still usable: the same fold without the flag gives the oracle factor
    R.zero_()
    status.zero_()
    rc = L.ifk_tsqr_fold(R.data_ptr(), n, 0, x.data_ptr(), n, rows, n, _lib.BF16, _lib.PREC_BF16, 0,
                         status.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert rel(R.cpu().numpy(), O.streaming_tsqr_update(None, X)) < 1e-2
