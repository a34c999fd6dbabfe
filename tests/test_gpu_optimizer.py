"""The drop-in optimizer and hooks on the GPU against trajectories recorded from the reference.

steps_c1: config 1 (Linear 128->256, ReLU, Linear 256->10, batch 256, cross-entropy,
lr 1e-3, damping 1e-2, factor refresh every step, momentum 0.9).
steps_sched: factor_update_freq 3 (plain-SGD warm-up without momentum and without
bias updates), momentum 0.5, weight decay 0.1, natural-gradient clip 0.5,
layers with and without bias, two alternating batches.
hooks_seq_bias: 3-D inputs flattened to rows (max_seq_rows=0) and the bias column.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from tests.golden_io import load, rel

pytestmark = pytest.mark.gpu


def _load_model(model, g):
    model.load_state_dict({k[5:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("init_")})
    return model.cuda()


def _run(model, opt, xs, ys, loss_fn, steps, record):
    out, losses = {}, []
    for s in range(1, steps + 1):
        x, y = xs[(s - 1) % len(xs)], ys[(s - 1) % len(ys)]
        loss = loss_fn(model(x), y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
        if s in record:
            for i, m in enumerate(opt.hooks.linear_layers):
                out[f"s{s}_W{i}"] = m.weight.detach().cpu().numpy().copy()
                if m.bias is not None:
                    out[f"s{s}_b{i}"] = m.bias.detach().cpu().numpy().copy()
    return out, np.array(losses)


def test_config1_trajectory_matches_reference():
    from ifkfac_b200 import IFKFAC
    g = load("steps_c1")
    model = _load_model(nn.Sequential(nn.Linear(128, 256), nn.ReLU(), nn.Linear(256, 10)), g)
    x = torch.from_numpy(g["x"]).cuda()
    y = torch.from_numpy(g["y"]).cuda()
    opt = IFKFAC(model, lr=1e-3, damping=1e-2, factor_update_freq=1, use_true_bf16=False)
    rec, losses = _run(model, opt, [x], [y], F.cross_entropy, 100, {1, 2, 10})
    for s, tol in ((1, 1e-5), (2, 1e-5), (10, 1e-4)):
        for k in ("W0", "b0", "W1", "b1"):
            e = rel(rec[f"s{s}_{k}"], g[f"s{s}_{k}"])
            assert e < tol, (s, k, e)
    ref = g["losses"]
    assert np.max(np.abs(losses[:20] - ref[:20]) / np.maximum(np.abs(ref[:20]), 1e-3)) < 1e-3
    assert losses[-1] < 1e-2 and ref[-1] < 1e-2   # both fit the batch
    opt.cleanup()


def test_schedule_trajectory_matches_reference():
    from ifkfac_b200 import IFKFAC
    g = load("steps_sched")
    model = _load_model(nn.Sequential(nn.Linear(24, 40), nn.Tanh(), nn.Linear(40, 16, bias=False), nn.Tanh(),
                                      nn.Linear(16, 8)), g)
    xs = [torch.from_numpy(g["x0"]).cuda(), torch.from_numpy(g["x1"]).cuda()]
    ys = [torch.from_numpy(g["y0"]).cuda(), torch.from_numpy(g["y1"]).cuda()]
    opt = IFKFAC(model, lr=2e-2, damping=1e-2, factor_update_freq=3, momentum=0.5, weight_decay=0.1,
                 grad_clip=0.5)
    rec, losses = _run(model, opt, xs, ys, F.mse_loss, 7, {1, 2, 3, 4, 6, 7})
    for s in (1, 2, 3, 4, 6, 7):
        for k in rec:
            if k.startswith(f"s{s}_"):
                e = rel(rec[k], g[k])
                assert e < 1e-5, (k, e)
    assert np.allclose(losses, g["losses"], rtol=1e-5)
    opt.cleanup()


def test_hooks_get_factors_3d_and_bias_column():
    from ifkfac_b200 import RawActivationHooks
    g = load("hooks_seq_bias")
    model = _load_model(nn.Sequential(nn.Linear(12, 20), nn.GELU(), nn.Linear(20, 6)), g)
    hooks = RawActivationHooks(model, damping=1e-3, augment_bias=True, max_seq_rows=0)
    hooks.enable()
    for k in range(3):
        model(torch.from_numpy(g[f"x{k}"]).cuda()).square().sum().backward()
    f = hooks.get_factors()
    for i, m in enumerate(hooks.linear_layers):
        assert [hooks._n_rows_X[m], hooks._n_rows_G[m]] == list(g[f"rows{i}"])
        assert rel(hooks._R_X[m].cpu().numpy(), g[f"rawRX{i}"]) < 1e-5
        assert rel(hooks._R_G[m].cpu().numpy(), g[f"rawRG{i}"]) < 1e-5
        assert rel(f[m][0].cpu().numpy(), g[f"RX{i}"]) < 1e-5
        assert rel(f[m][1].cpu().numpy(), g[f"RG{i}"]) < 1e-5
    hooks.remove()


def test_bf16_autocast_capture_runs_on_tensor_cores():
    """Under bf16 autocast the captured chunks are bf16: the reference's geqrf has no bf16
    kernel, here they fold on the tensor cores; compare with the fp32 upcast through the oracle."""
    from ifkfac_b200 import IFKFAC
    from oracle import ifk_oracle as O
    torch.manual_seed(3)
    model = nn.Sequential(nn.Linear(256, 384), nn.ReLU(), nn.Linear(384, 128)).cuda()
    opt = IFKFAC(model, lr=1e-3, damping=1e-2, factor_update_freq=1, use_true_bf16=True)
    caps = []
    # the first layer sees the fp32 input (autocast casts inside the op); the second sees bf16
    h = model[2].register_forward_hook(lambda m, i, o: caps.append(i[0].detach().clone()))
    x = torch.randn(1024, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(x).float().square().mean()
    loss.backward()
    h.remove()
    f = opt.hooks.get_factors()
    RX = f[model[2]][0].cpu().numpy()
    Xc = caps[0].float().cpu().numpy()
    assert caps[0].dtype == torch.bfloat16
    want = O.get_factor(O.streaming_tsqr_update(None, Xc), Xc.shape[0], 1e-2)
    assert rel(RX, want) < 1e-2
    opt.step()
    assert all(v[0].dtype == torch.bfloat16 for v in opt._factors.values())
    opt.cleanup()


def test_ema_blend_trajectory_matches_reference():
    """gamma = 0.4, refresh every 2 steps: the step-4 factors are the exact blend of the
    reference (ifkfac/ifkfac.py:261-285) and the weights follow its trajectory."""
    from ifkfac_b200 import IFKFAC
    g = load("ema_blend")
    model = _load_model(nn.Sequential(nn.Linear(20, 24), nn.ReLU(), nn.Linear(24, 5)), g)
    x = torch.from_numpy(g["x"]).cuda()
    y = torch.from_numpy(g["y"]).cuda()
    opt = IFKFAC(model, lr=5e-2, damping=1e-2, factor_update_freq=2, momentum=0.9, gamma=0.4)
    for s in range(1, 5):
        loss = F.cross_entropy(model(x), y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        if s in (2, 4):
            for i, m in enumerate(opt.hooks.linear_layers):
                for j, f in enumerate(("RX", "RG")):
                    e = rel(opt._factors[m][j].cpu().numpy(), g[f"ema_s{s}_{f}{i}"])
                    assert e < 1e-4, (s, i, f, e)
    for i, m in enumerate(opt.hooks.linear_layers):
        e = rel(m.weight.detach().cpu().numpy(), g[f"ema_W{i}"])
        assert e < 1e-4, (i, e)
    opt.cleanup()


def test_nonfinite_factor_skips_only_its_layer():
    """A refresh finalizes every layer in shared launches; a layer whose factor is not
    finite is skipped on its own (ifkfac/ifkfac.py:231-237) while the others get
    their factors, and the skipped layer takes the plain gradient step."""
    from ifkfac_b200 import IFKFAC
    torch.manual_seed(5)
    model = nn.Sequential(nn.Linear(16, 32), nn.ReLU(), nn.Linear(32, 32), nn.ReLU(), nn.Linear(32, 4)).cuda()
    x = torch.randn(128, 16, device="cuda")
    y = torch.randint(0, 4, (128,), device="cuda")
    opt = IFKFAC(model, lr=1e-2, damping=1e-2, factor_update_freq=1, momentum=0.0)
    layers = opt.hooks.linear_layers
    loss = F.cross_entropy(model(x), y)
    opt.zero_grad()
    loss.backward()
    opt.hooks._fx[layers[1]].R[0, 0] = float("nan")  # the running factor of layer 1 goes bad
    w1 = layers[1].weight.detach().clone()
    g1 = layers[1].weight.grad.detach().clone()
    opt.step()
    torch.cuda.synchronize()
    assert layers[0] in opt._factors and layers[2] in opt._factors
    assert layers[1] not in opt._factors
    for m in (layers[0], layers[2]):
        for R in opt._factors[m]:
            assert torch.isfinite(R).all()
    # no preconditioner for layer 1: plain SGD on its weight (ifkfac/ifkfac.py:443-448)
    assert torch.allclose(layers[1].weight.detach(), w1 - 1e-2 * g1, rtol=0, atol=1e-7)
    opt.cleanup()
