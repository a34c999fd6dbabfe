"""Host-side logic of the front end, on CPU (no GPU work): chunk preprocessing,
refresh schedule, layer selection and the constructor contract of the reference."""
import inspect

import numpy as np
import pytest
import torch
import torch.nn as nn

from ifkfac_b200 import activation_hooks as AH
from ifkfac_b200.ifkfac import IFKFAC, should_refresh
from oracle import ifk_oracle as O


def test_refresh_schedule_matches_oracle():
    for freq in (1, 2, 3, 10):
        assert [should_refresh(s, freq) for s in range(1, 41)] == [O.should_refresh(s, freq) for s in range(1, 41)]


def test_prepare_x_sequence_flatten_bias_and_subsample():
    lin = nn.Linear(6, 4)
    x = torch.randn(2, 5, 6)
    r = AH.prepare_x(x, lin, 512, 0, True)
    assert (r.rows, r.cols, r.ones, r.index) == (10, 7, True, None)
    assert r.x.data_ptr() == x.data_ptr()             # the 3-D reshape is a view: nothing copied
    c = r.materialize()
    assert c.shape == (10, 7) and torch.all(c[:, -1] == 1)
    assert torch.equal(c[:, :6], x.reshape(-1, 6))
    torch.manual_seed(0)
    r2 = AH.prepare_x(x, lin, 512, 4, False)          # randperm row subsample to max_seq_rows
    assert r2.rows == 4 and r2.cols == 6 and r2.x.data_ptr() == x.data_ptr()
    torch.manual_seed(0)
    assert torch.equal(r2.index, torch.randperm(10)[:4])   # the reference's draw, kept as indices
    rows = {tuple(t.tolist()) for t in x.reshape(-1, 6)}
    assert all(tuple(t.tolist()) in rows for t in r2.materialize())
    assert AH.prepare_x(torch.randn(3, 6), nn.Linear(6, 4, bias=False), 512, 0, True).cols == 6
    # a chunk transform sees the materialised rows and its output is folded
    t = AH.prepare_x(x, lin, 512, 0, True, transform=lambda m: m * 2)
    assert torch.is_tensor(t) and torch.equal(t, 2 * c)


def test_prepare_conv_im2col_and_grad_layout():
    conv = nn.Conv2d(3, 5, kernel_size=3, padding=1)
    x = torch.randn(2, 3, 4, 4)
    c = AH.prepare_x(x, conv, 0, 0, False).materialize()
    assert c.shape == (2 * 16, 3 * 9)
    d = torch.randn(2, 5, 4, 4)
    g = AH.prepare_g(d, conv, 0).materialize()
    assert g.shape == (32, 5) and torch.equal(g[0], d[0, :, 0, 0])
    assert AH.prepare_x(x, conv, 8, 0, False).rows == 8                  # max_conv_rows cap


def test_layer_selection_and_constructor_contract():
    model = nn.Sequential(nn.Linear(8, 16), nn.ReLU(), nn.Linear(16, 5000), nn.Conv2d(1, 2, 3))
    hooks = AH.RawActivationHooks(model, max_out_dim=4096)
    assert hooks.linear_layers == [model[0], model[3]]             # the 5000-wide head is skipped
    with pytest.raises(ValueError):
        AH.RawActivationHooks(model, batched=True, deferred=True)
    sig = inspect.signature(IFKFAC.__init__)
    for name, default in (("lr", 1e-3), ("damping", 1e-2), ("factor_update_freq", 10), ("weight_decay", 0.0),
                          ("momentum", 0.9), ("grad_clip", None), ("gamma", 0.0), ("max_out_dim", 0),
                          ("augment_bias", False), ("max_conv_rows", 512), ("max_seq_rows", None),
                          ("batched_qr", False), ("deferred_qr", False), ("use_true_bf16", False)):
        assert sig.parameters[name].default == default, name


def test_cpu_tensors_are_refused():
    """No CPU path: folding a CPU chunk raises instead of computing anything."""
    model = nn.Sequential(nn.Linear(4, 3))
    hooks = AH.RawActivationHooks(model)
    hooks.enable()
    with pytest.raises(ValueError, match="CUDA"):
        model(torch.randn(8, 4))
    hooks.remove()
