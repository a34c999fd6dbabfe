"""Generate the golden vectors in this folder by running the reference on CPU.

Usage (in a container where the reference source tree is available):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref <path-to-reference>

The reference (Gsend/ifkfac) is pure Python on PyTorch; this script imports
it, runs the functions on the curvature path on small seeded inputs and saves
inputs and outputs as compressed .npz files.  The files are committed; tests
only read them and never import the reference.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    # a copy: .numpy() of a CPU tensor shares its storage, and parameters keep changing
    t = t.detach().cpu()
    return (t.float() if t.dtype == torch.bfloat16 else t).numpy().copy()


def _scaled(g, p, n, dtype, lo=0.0, hi=math.log(100.0)):
    s = torch.exp(torch.empty(n, dtype=torch.float64).uniform_(lo, hi, generator=g))
    return (torch.randn(p, n, generator=g, dtype=torch.float64) * s).to(dtype)


def gen_streaming(T):
    out = {}
    for dtype, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
        g = torch.Generator().manual_seed(11)
        n = 48
        rows = [20, 30, 64, 7, 100]
        R = None
        total = 0
        for i, r in enumerate(rows):
            chunk = _scaled(g, r, n, dtype)
            R = T.streaming_tsqr_update(R, chunk)
            total += r
            out[f"{tag}_chunk{i}"] = _np(chunk)
            out[f"{tag}_R{i}"] = _np(R)
        out[f"{tag}_rows"] = np.array(rows)
        Rs = R / math.sqrt(total)
        out[f"{tag}_final"] = _np(T.finalize_R(Rs, 1e-2))
        out[f"{tag}_final_l3"] = _np(T.finalize_R(Rs, 1e-3))
    np.savez_compressed(os.path.join(HERE, "streaming_tsqr.npz"), **out)


def gen_apply(T):
    out = {}
    for dtype, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
        g = torch.Generator().manual_seed(12)
        n_in, n_out, p = 40, 24, 160
        X = _scaled(g, p, n_in, dtype)
        D = _scaled(g, p, n_out, dtype)
        RX = T.finalize_R(T.streaming_tsqr_update(None, X) / math.sqrt(p), 1e-2)
        RG = T.finalize_R(T.streaming_tsqr_update(None, D) / math.sqrt(p), 1e-2)
        gW = torch.randn(n_out, n_in, generator=g, dtype=dtype) * 1e-2
        gb = torch.randn(n_out, generator=g, dtype=dtype) * 1e-2
        out[f"{tag}_RX"], out[f"{tag}_RG"] = _np(RX), _np(RG)
        out[f"{tag}_gW"], out[f"{tag}_gb"] = _np(gW), _np(gb)
        out[f"{tag}_nat"] = _np(T.apply_vered(gW, RX, RG))
        out[f"{tag}_natb"] = _np(T.apply_vered_bias(gb, RG))
        if dtype == torch.float32:
            RXb, RGb = RX.bfloat16(), RG.bfloat16()
            out["bf16_RX"], out["bf16_RG"] = _np(RXb), _np(RGb)
            out["bf16_nat"] = _np(T.apply_vered(gW, RXb, RGb))
            out["bf16_natb"] = _np(T.apply_vered_bias(gb, RGb))
            Bst = 3
            gWs = torch.randn(Bst, n_out, n_in, generator=g, dtype=dtype)
            out["batched_gW"] = _np(gWs)
            out["batched_nat"] = _np(T.apply_vered_batched(
                gWs, RX.expand(Bst, -1, -1).contiguous(), RG.expand(Bst, -1, -1).contiguous()))
    np.savez_compressed(os.path.join(HERE, "apply_vered.npz"), **out)


def gen_batched_and_tree(T):
    g = torch.Generator().manual_seed(13)
    B, p, n = 3, 16, 12
    chunks = torch.randn(B, p, n, generator=g)
    running = torch.zeros(B, n, n)
    running[1] = T.streaming_tsqr_update(None, torch.randn(30, n, generator=g))
    outb = T.batched_streaming_tsqr_update(running, chunks)
    M = _scaled(g, 200, 24, torch.float64)
    np.savez_compressed(os.path.join(HERE, "batched_tree.npz"),
                        chunks=_np(chunks), running=_np(running), out=_np(outb),
                        M=_np(M), tree64=_np(T.tsqr(M, 64)), tree200=_np(T.tsqr(M, 512)))


def gen_bf16(B):
    out = {}
    g = torch.Generator().manual_seed(14)
    for (m, n, bs, tag) in ((256, 64, 32, "a"), (96, 40, 16, "b")):
        A = _scaled(g, m, n, torch.float32).bfloat16()
        out[f"qr_{tag}_A"] = _np(A)
        out[f"qr_{tag}_R"] = _np(B.block_householder_qr_bf16(A, bs))
        out[f"qr_{tag}_bs"] = np.array(bs)
    Rt = torch.triu(torch.randn(32, 32, generator=g)) + 3 * torch.eye(32)
    Bm = torch.randn(32, 8, generator=g)
    out["tri_R"] = _np(Rt.bfloat16())
    out["tri_B"] = _np(Bm.bfloat16())
    out["tri_up"] = _np(B.solve_triangular_bf16(Rt.bfloat16(), Bm.bfloat16(), upper=True))
    out["tri_lo"] = _np(B.solve_triangular_bf16(Rt.t().contiguous().bfloat16(), Bm.bfloat16(), upper=False))
    # composition used as the bf16 oracle: p=256, n=64, kappa ~ 1e2 from column scales
    p, n, lam = 256, 64, 1e-2
    X = _scaled(g, p, n, torch.float32).bfloat16()
    D = _scaled(g, p, n, torch.float32).bfloat16()
    gW = (torch.randn(n, n, generator=g) * 1e-2)

    def factor(A):
        R = B.block_householder_qr_bf16(A, 32).float()
        s = torch.sign(torch.diagonal(R)); s[s == 0] = 1
        R = (R * s[:, None]).bfloat16() / math.sqrt(p)
        aug = torch.cat([R, (math.sqrt(lam) * torch.eye(n)).bfloat16()], 0)
        R2 = B.block_householder_qr_bf16(aug, 32).float()
        s = torch.sign(torch.diagonal(R2)); s[s == 0] = 1
        return (R2 * s[:, None]).bfloat16()

    RX, RG = factor(X), factor(D)
    gb = gW.bfloat16()
    t1 = B.solve_triangular_bf16(RG.t().contiguous(), gb, upper=False)
    t2 = B.solve_triangular_bf16(RG, t1, upper=True)
    t3 = B.solve_triangular_bf16(RX.t().contiguous(), t2.t().contiguous(), upper=False)
    t4 = B.solve_triangular_bf16(RX, t3, upper=True)
    out.update(comp_X=_np(X), comp_D=_np(D), comp_gW=_np(gW), comp_RX=_np(RX), comp_RG=_np(RG),
               comp_nat=_np(t4.t().contiguous()), comp_lam=np.array(lam))
    np.savez_compressed(os.path.join(HERE, "bf16_linalg.npz"), **out)


def _run_ifkfac(ifk, model, xs, ys, loss_fn, steps, record, **kw):
    opt = ifk.IFKFAC(model, **kw)
    rec = {}
    losses = []
    with contextlib.redirect_stdout(io.StringIO()):
        for s in range(1, steps + 1):
            x, y = xs[(s - 1) % len(xs)], ys[(s - 1) % len(ys)]
            loss = loss_fn(model(x), y)
            opt.zero_grad()
            loss.backward()
            opt.step()
            losses.append(float(loss.detach()))
            if s in record:
                for i, m in enumerate(opt.hooks.linear_layers):
                    rec[f"s{s}_W{i}"] = _np(m.weight)
                    if m.bias is not None:
                        rec[f"s{s}_b{i}"] = _np(m.bias)
    opt.cleanup()
    rec["losses"] = np.array(losses)
    return rec


def gen_steps(ifk):
    import torch.nn as nn
    import torch.nn.functional as F
    # config 1 shape: Linear(128->256)-ReLU-Linear(256->10), batch 256, CE, freq 1
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(128, 256), nn.ReLU(), nn.Linear(256, 10))
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 128, generator=g)
    y = torch.randint(0, 10, (256,), generator=g)
    init = {f"init_{k}": v.detach().numpy().copy() for k, v in model.state_dict().items()}
    rec = _run_ifkfac(ifk, model, [x], [y], F.cross_entropy, 100, {1, 2, 10},
                      lr=1e-3, damping=1e-2, factor_update_freq=1, use_true_bf16=False)
    np.savez_compressed(os.path.join(HERE, "steps_c1.npz"), x=x.numpy(), y=y.numpy(), **init, **rec)
    # schedule coverage: freq 3 (SGD warm-up, no momentum before the first refresh),
    # weight decay, grad clip, bias, two alternating batches, MSE loss.
    torch.manual_seed(1)
    model = nn.Sequential(nn.Linear(24, 40), nn.Tanh(), nn.Linear(40, 16, bias=False), nn.Tanh(),
                          nn.Linear(16, 8))
    g = torch.Generator().manual_seed(1)
    xs = [torch.randn(64, 24, generator=g) for _ in range(2)]
    ys = [torch.randn(64, 8, generator=g) for _ in range(2)]
    init = {f"init_{k}": v.detach().numpy().copy() for k, v in model.state_dict().items()}
    rec = _run_ifkfac(ifk, model, xs, ys, F.mse_loss, 7, {1, 2, 3, 4, 6, 7},
                      lr=2e-2, damping=1e-2, factor_update_freq=3, momentum=0.5,
                      weight_decay=0.1, grad_clip=0.5)
    np.savez_compressed(os.path.join(HERE, "steps_sched.npz"),
                        x0=xs[0].numpy(), x1=xs[1].numpy(), y0=ys[0].numpy(), y1=ys[1].numpy(),
                        **init, **rec)


def gen_hooks(ifk):
    import torch.nn as nn
    torch.manual_seed(2)
    model = nn.Sequential(nn.Linear(12, 20), nn.GELU(), nn.Linear(20, 6))
    hooks = ifk.RawActivationHooks(model, damping=1e-3, augment_bias=True, max_seq_rows=0)
    hooks.enable()
    g = torch.Generator().manual_seed(2)
    xs = [torch.randn(3, 5, 12, generator=g) for _ in range(3)]   # (B, T, d): 15 rows per call
    init = {f"init_{k}": v.detach().numpy().copy() for k, v in model.state_dict().items()}
    for x in xs:
        model(x).square().sum().backward()
    f = hooks.get_factors()
    out = {f"x{i}": x.numpy() for i, x in enumerate(xs)}
    for i, m in enumerate(hooks.linear_layers):
        out[f"RX{i}"], out[f"RG{i}"] = _np(f[m][0]), _np(f[m][1])
        out[f"rawRX{i}"], out[f"rawRG{i}"] = _np(hooks._R_X[m]), _np(hooks._R_G[m])
        out[f"rows{i}"] = np.array([hooks._n_rows_X[m], hooks._n_rows_G[m]])
    hooks.remove()
    np.savez_compressed(os.path.join(HERE, "hooks_seq_bias.npz"), **init, **out)


def gen_ema(ifk):
    """EMA blend (ifkfac/ifkfac.py:261-285): freq 2, gamma 0.4, so the refresh of
    step 4 blends with the factors of step 2.  A second run with gamma 0 from the
    same start gives the unblended step-4 factors (steps 1-3 do not depend on gamma)."""
    import torch.nn as nn
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(4)
    x = torch.randn(64, 20, generator=g)
    y = torch.randint(0, 5, (64,), generator=g)
    torch.manual_seed(4)
    init_model = nn.Sequential(nn.Linear(20, 24), nn.ReLU(), nn.Linear(24, 5))
    init = {f"init_{k}": v.detach().numpy().copy() for k, v in init_model.state_dict().items()}
    out = {"x": x.numpy(), "y": y.numpy(), **init}
    for gamma, tag in ((0.4, "ema"), (0.0, "plain")):
        model = nn.Sequential(nn.Linear(20, 24), nn.ReLU(), nn.Linear(24, 5))
        model.load_state_dict(init_model.state_dict())
        opt = ifk.IFKFAC(model, lr=5e-2, damping=1e-2, factor_update_freq=2, momentum=0.9, gamma=gamma)
        with contextlib.redirect_stdout(io.StringIO()):
            for s in range(1, 5):
                loss = F.cross_entropy(model(x), y)
                opt.zero_grad()
                loss.backward()
                opt.step()
                if s in (2, 4):
                    for i, m in enumerate(opt.hooks.linear_layers):
                        out[f"{tag}_s{s}_RX{i}"] = _np(opt._factors[m][0])
                        out[f"{tag}_s{s}_RG{i}"] = _np(opt._factors[m][1])
        for i, m in enumerate(opt.hooks.linear_layers):
            out[f"{tag}_W{i}"] = _np(m.weight)
        opt.cleanup()
    np.savez_compressed(os.path.join(HERE, "ema_blend.npz"), **out)


def gen_laplace(ifk):
    """K-FAC Laplace draw (ifkfac/laplace.py:58-149): two layers whose EVD
    factors come from svd(R) (A = R^T R: U_A = right singular vectors, d_A =
    squared singular values, :27-29), prior precision 0.5, N = 100.  The draw's
    xi are replayed from the same seeded generator in the reference's order."""
    import torch.nn as nn
    g = torch.Generator().manual_seed(11)
    torch.manual_seed(11)
    model = nn.Sequential(nn.Linear(12, 16), nn.ReLU(), nn.Linear(16, 6))
    layers = [model[0], model[2]]
    N, lam = 100, 0.5
    out = {"N": np.array(N), "lam": np.array(lam)}
    evd = {}
    for i, m in enumerate(layers):
        n_out, n_in = m.weight.shape
        for tag, n in (("A", n_in), ("G", n_out)):
            Xs = _scaled(g, 3 * n, n, torch.float32)
            R = torch.linalg.qr(Xs, mode="r")[1]
            R = R * torch.sign(torch.diagonal(R)).unsqueeze(1)
            _, sv, Vh = torch.linalg.svd(R)
            out[f"R_{tag}{i}"], out[f"U_{tag}{i}"], out[f"d_{tag}{i}"] = _np(R), _np(Vh.T), _np(sv ** 2)
        evd[m] = (torch.from_numpy(out[f"U_A{i}"]), torch.from_numpy(out[f"d_A{i}"]),
                  torch.from_numpy(out[f"U_G{i}"]), torch.from_numpy(out[f"d_G{i}"]))
        out[f"Wmap{i}"] = _np(m.weight)
    post = ifk.LaplacePosterior(model, evd, prior_precision=lam, dataset_size=N)
    with contextlib.redirect_stdout(io.StringIO()):
        post.sample_in_place(generator=torch.Generator().manual_seed(5))
    replay = torch.Generator().manual_seed(5)
    for i, m in enumerate(layers):
        out[f"xi{i}"] = _np(torch.randn(*m.weight.shape, dtype=torch.float32, generator=replay))
        out[f"Wsample{i}"] = _np(m.weight)
    np.savez_compressed(os.path.join(HERE, "laplace.npz"), **out)


def gen_classic(ifk):
    """ClassicKFAC (ifkfac/classic_kfac.py) trajectories on CPU: an MLP with weight
    decay, momentum and an EMA of the Gram factors (freq 2, decomp freq 2), and a
    small conv net (im2col factors, kfac_hooks.py:151-174); parameters after every
    step."""
    import torch.nn as nn
    import torch.nn.functional as F
    out = {}
    g = torch.Generator().manual_seed(21)
    cases = {
        "mlp": (lambda: nn.Sequential(nn.Linear(10, 14), nn.Tanh(), nn.Linear(14, 4)),
                torch.randn(48, 10, generator=g), torch.randint(0, 4, (48,), generator=g)),
        "conv": (lambda: nn.Sequential(nn.Conv2d(2, 3, 3, padding=1), nn.ReLU(), nn.Flatten(), nn.Linear(3 * 25, 4)),
                 torch.randn(16, 2, 5, 5, generator=g), torch.randint(0, 4, (16,), generator=g)),
    }
    for tag, (make, x, y) in cases.items():
        torch.manual_seed(21)
        model = make()
        out[f"{tag}_x"], out[f"{tag}_y"] = x.numpy(), y.numpy()
        for k, v in model.state_dict().items():
            out[f"{tag}_init_{k}"] = v.numpy().copy()
        opt = ifk.ClassicKFAC(model, lr=5e-2, damping=1e-2, factor_update_freq=2, decomp_update_freq=2,
                              weight_decay=1e-3, momentum=0.9, gamma=0.3)
        for s in range(1, 6):
            loss = F.cross_entropy(model(x), y)
            opt.zero_grad()
            loss.backward()
            opt.step()
            for k, v in model.state_dict().items():
                out[f"{tag}_s{s}_{k}"] = v.numpy().copy()
        opt.cleanup()
    np.savez_compressed(os.path.join(HERE, "classic.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference source tree")
    ap.add_argument("--only", default=None, help="write one file: streaming, apply, batched, bf16, steps, hooks, ema, laplace, classic")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import ifkfac as ifk
    from ifkfac import triangular as T, bf16_linalg as B
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    gens = {"streaming": lambda: gen_streaming(T), "apply": lambda: gen_apply(T),
            "batched": lambda: gen_batched_and_tree(T), "bf16": lambda: gen_bf16(B),
            "steps": lambda: gen_steps(ifk), "hooks": lambda: gen_hooks(ifk), "ema": lambda: gen_ema(ifk),
            "laplace": lambda: gen_laplace(ifk), "classic": lambda: gen_classic(ifk)}
    for name, gen in gens.items():
        if args.only in (None, name):
            gen()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
