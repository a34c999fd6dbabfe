"""Batched natural gradient (ifk_natgrad_batched): the layers of one call share
the inverse, pack and solve launches, and each layer's result is bit for bit
the one of ifk_natgrad; the optimizer's batched apply gives the weights of the
per-layer apply."""
import copy
import ctypes
import math

import pytest
import torch

from ifkfac_b200 import _lib

pytestmark = pytest.mark.gpu


def _factor(n, seed, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = torch.exp(torch.rand(n, generator=g, device="cuda") * math.log(100.0))
    X = torch.randn(3 * n, n, generator=g, device="cuda") * s
    R = torch.linalg.qr(X.double().cpu(), mode="r")[1]
    R = R * torch.sign(torch.diagonal(R)).unsqueeze(1)
    R = torch.linalg.qr(torch.cat([R / math.sqrt(3 * n), 0.1 * torch.eye(n, dtype=R.dtype)]), mode="r")[1]
    R = R * torch.sign(torch.diagonal(R)).unsqueeze(1)
    return R.to(device="cuda", dtype=dtype).contiguous()


def _single(g, RX, RG, prec):
    L = _lib.lib()
    n_out, n_in = g.shape
    nat = torch.empty_like(g)
    ws = torch.empty(L.ifk_natgrad_workspace(n_out, n_in), dtype=torch.uint8, device="cuda")
    _lib.check(L.ifk_natgrad(g.data_ptr(), n_in, RX.data_ptr(), n_in, RG.data_ptr(), n_out,
                             _lib.BF16 if RX.dtype == torch.bfloat16 else _lib.F32, nat.data_ptr(), n_in, n_out,
                             n_in, prec, None, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream),
               "ifk_natgrad")
    return nat


def _batched(gs, RXs, RGs, prec, bias=None):
    L = _lib.lib()
    arr = lambda t, v: (t * len(v))(*v)
    n_out = [g.shape[0] for g in gs]
    n_in = [g.shape[1] for g in gs]
    nats = [torch.empty_like(g) for g in gs]
    nbs = [torch.empty_like(b) if b is not None else None for b in bias] if bias else None
    ws = torch.empty(L.ifk_natgrad_batched_workspace(len(gs), arr(ctypes.c_int64, n_out), arr(ctypes.c_int64, n_in)),
                     dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(L.ifk_natgrad_batched(
        len(gs), arr(ctypes.c_void_p, [g.data_ptr() for g in gs]), arr(ctypes.c_int64, n_in),
        arr(ctypes.c_void_p, [r.data_ptr() for r in RXs]), arr(ctypes.c_int64, n_in),
        arr(ctypes.c_void_p, [r.data_ptr() for r in RGs]), arr(ctypes.c_int64, n_out),
        _lib.BF16 if RXs[0].dtype == torch.bfloat16 else _lib.F32, arr(ctypes.c_void_p, [o.data_ptr() for o in nats]),
        arr(ctypes.c_int64, n_in), arr(ctypes.c_int64, n_out), arr(ctypes.c_int64, n_in),
        arr(ctypes.c_void_p, [b.data_ptr() if b is not None else None for b in bias]) if bias else None,
        arr(ctypes.c_void_p, [b.data_ptr() if b is not None else None for b in nbs]) if bias else None,
        prec, st.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream),
        "ifk_natgrad_batched")
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    return (nats, nbs) if bias else nats


@pytest.mark.parametrize("dtype,prec", [(torch.bfloat16, _lib.PREC_BF16), (torch.float32, _lib.PREC_FP32)])
def test_batched_equals_per_layer(dtype, prec):
    # ragged orders, a factor order that is not a multiple of 8 (per-layer path), tall and wide layers
    shapes = [(136, 264), (1000, 520), (256, 8), (640, 384), (300, 300), (2048, 1024), (130, 97)]
    gs, RXs, RGs = [], [], []
    for i, (n_out, n_in) in enumerate(shapes):
        RXs.append(_factor(n_in, 10 + i, dtype))
        RGs.append(_factor(n_out, 50 + i, dtype))
        g = torch.Generator(device="cuda").manual_seed(90 + i)
        gs.append(torch.randn(n_out, n_in, generator=g, device="cuda") * 1e-2)
    nats = _batched(gs, RXs, RGs, prec)
    for g, RX, RG, nat in zip(gs, RXs, RGs, nats):
        ref = _single(g, RX, RG, prec)
        torch.cuda.synchronize()
        assert torch.equal(nat, ref), float((nat - ref).abs().max())


def test_batched_many_layers_over_several_launches():
    """More layers than one launch's problem table (64) run as several groups."""
    shapes = [(128 + 8 * (i % 5), 136 + 8 * (i % 3)) for i in range(70)]
    gs, RXs, RGs = [], [], []
    for i, (n_out, n_in) in enumerate(shapes):
        RXs.append(_factor(n_in, 200 + i, torch.bfloat16))
        RGs.append(_factor(n_out, 400 + i, torch.bfloat16))
        gs.append(torch.randn(n_out, n_in, device="cuda") * 1e-2)
    nats = _batched(gs, RXs, RGs, _lib.PREC_BF16)
    for k in (0, 33, 63, 64, 69):
        ref = _single(gs[k], RXs[k], RGs[k], _lib.PREC_BF16)
        torch.cuda.synchronize()
        assert torch.equal(nats[k], ref)


@pytest.mark.parametrize("bias", [False, True])
def test_optimizer_batched_apply_equals_per_layer(bias):
    """Without biases the batched apply gives the per-layer weights bit for bit; with
    biases their solves run on the tensor cores beside the weights' (the per-layer
    bias solve is fp32), so the trajectories agree to the bf16 mode's accuracy."""
    from ifkfac_b200.ifkfac import IFKFAC
    torch.manual_seed(0)
    base = torch.nn.Sequential(torch.nn.Linear(256, 512, bias=bias), torch.nn.ReLU(),
                               torch.nn.Linear(512, 512, bias=bias), torch.nn.ReLU(),
                               torch.nn.Linear(512, 128, bias=bias)).cuda()
    x = torch.randn(1024, 256, device="cuda")
    y = torch.randint(0, 128, (1024,), device="cuda")
    weights = []
    for batched in (True, False):
        model = copy.deepcopy(base)
        opt = IFKFAC(model, lr=1e-2, damping=1e-2, factor_update_freq=1, momentum=0.9, use_true_bf16=True)
        if not batched:
            opt._batched_natgrads = lambda modules: {}
        for _ in range(3):
            opt.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = model(x)
            torch.nn.functional.cross_entropy(out.float(), y).backward()
            opt.step()
        torch.cuda.synchronize()
        weights.append([p.detach().clone() for p in model.parameters()])
        opt.cleanup()
    for a, b in zip(*weights):
        if bias:
            assert float((a - b).norm() / a.norm()) < 1e-3
        else:
            assert torch.equal(a, b), float((a - b).abs().max())


def test_batched_bias_solves():
    """Biases ride along as one more right-hand side of the left solves: R_G^-1 R_G^-T g_b,
    held to the fp64 solve with the same factor (bf16 mode) and to ifk_natgrad_bias."""
    L = _lib.lib()
    shapes = [(136, 264), (1000, 520), (2048, 1024), (130, 97)]
    gs, RXs, RGs, bs = [], [], [], []
    for i, (n_out, n_in) in enumerate(shapes):
        RXs.append(_factor(n_in, 10 + i, torch.bfloat16))
        RGs.append(_factor(n_out, 50 + i, torch.bfloat16))
        gs.append(torch.randn(n_out, n_in, device="cuda") * 1e-2)
        bs.append(torch.randn(n_out, device="cuda") * 1e-2 if i != 1 else None)
    nats, nbs = _batched(gs, RXs, RGs, _lib.PREC_BF16, bias=bs)
    for i, (RG, b, nb) in enumerate(zip(RGs, bs, nbs)):
        if b is None:
            assert nb is None
            continue
        R = RG.double()
        truth = torch.linalg.solve_triangular(R, torch.linalg.solve_triangular(R.T, b.double()[:, None], upper=False),
                                              upper=True)[:, 0]
        rel = float((nb.double() - truth).norm() / truth.norm())
        assert rel < 5e-3, (i, rel)
        single = torch.empty_like(b)
        _lib.check(L.ifk_natgrad_bias(b.data_ptr(), RG.data_ptr(), RG.shape[0], _lib.BF16, single.data_ptr(),
                                      RG.shape[0], _lib.PREC_BF16, None, 0, torch.cuda.current_stream().cuda_stream),
                   "ifk_natgrad_bias")
        torch.cuda.synchronize()
        assert float((nb - single).norm() / single.norm()) < 5e-3
    # the weights are unchanged by the bias problems sharing their launches
    for g, RX, RG, nat in zip(gs, RXs, RGs, nats):
        assert torch.equal(nat, _single(g, RX, RG, _lib.PREC_BF16))


@pytest.mark.parametrize("prec,tol", [(_lib.PREC_FP32, 1e-5), (_lib.PREC_BF16, 2e-2)])
def test_ema_blend_matches_oracle(prec, tol):
    """IFKFAC(gamma > 0) blends refreshed factors by the exact stacked QR of the
    reference (ifkfac/ifkfac.py:261-285): fold sqrt(1-g) R_new into sqrt(g) R_old."""
    import numpy as np
    from oracle import ifk_oracle as ora
    from ifkfac_b200.ifkfac import IFKFAC
    model = torch.nn.Sequential(torch.nn.Linear(8, 8)).cuda()
    opt = IFKFAC(model, gamma=0.3, precision=prec)
    for n in (96, 200):
        R_old = _factor(n, 1 + n, torch.float32)
        R_new = _factor(n, 2 + n, torch.float32)
        out = opt._blend(R_old, R_new).double().cpu().numpy()
        truth = ora.ema_blend(R_old.double().cpu().numpy(), R_new.double().cpu().numpy(), 0.3)
        assert np.linalg.norm(out - truth) / np.linalg.norm(truth) < tol
        G = 0.3 * R_old.double().T @ R_old.double() + 0.7 * R_new.double().T @ R_new.double()
        assert float(np.linalg.norm(out.T @ out - G.cpu().numpy()) / np.linalg.norm(G.cpu().numpy())) < 2 * tol
    opt.cleanup()


@pytest.mark.parametrize("n_out,n_in", [(100, 2048), (10, 256), (3, 5), (1000, 1001), (2047, 96)])
def test_padded_orders_on_the_persistent_solves(n_out, n_in):
    """Orders that are not multiples of 8 solve on [[R, 0], [0, I]] padded to the next
    multiple of 8 with a zero-padded right-hand side: the leading block is the natural
    gradient (held to the fp64 solve with the same bf16 factors), in both entry points
    bit for bit."""
    RX, RG = _factor(n_in, 3 + n_in, torch.bfloat16), _factor(n_out, 5 + n_out, torch.bfloat16)
    g = torch.randn(n_out, n_in, generator=torch.Generator(device="cuda").manual_seed(n_out), device="cuda")
    one = _single(g, RX, RG, _lib.PREC_BF16)
    many = _batched([g], [RX], [RG], _lib.PREC_BF16)[0]
    torch.cuda.synchronize()
    assert torch.equal(one, many)
    X, G = RX.double(), RG.double()
    t = torch.linalg.solve_triangular(G, torch.linalg.solve_triangular(G.T, g.double(), upper=False), upper=True)
    truth = torch.linalg.solve_triangular(X, torch.linalg.solve_triangular(X.T, t.T, upper=False), upper=True).T
    rel = float((one.double() - truth).norm() / truth.norm())
    assert rel < 5e-3, rel
