"""Classic K-FAC comparator (ifkfac/classic_kfac.py, ifkfac/kfac_hooks.py) on the
CPU: its trajectories follow the reference's own (golden classic.npz: an MLP with
weight decay, momentum and the Gram EMA; a conv net through im2col)."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from ifkfac_b200.classic_kfac import ClassicKFAC
from tests.golden_io import load, rel

CASES = {
    "mlp": lambda: nn.Sequential(nn.Linear(10, 14), nn.Tanh(), nn.Linear(14, 4)),
    "conv": lambda: nn.Sequential(nn.Conv2d(2, 3, 3, padding=1), nn.ReLU(), nn.Flatten(), nn.Linear(3 * 25, 4)),
}


def run_classic(tag, device):
    g = load("classic")
    model = CASES[tag]().to(device)
    model.load_state_dict({k: torch.from_numpy(g[f"{tag}_init_{k}"]) for k in model.state_dict()})
    x = torch.from_numpy(g[f"{tag}_x"]).to(device)
    y = torch.from_numpy(g[f"{tag}_y"]).to(device)
    opt = ClassicKFAC(model, lr=5e-2, damping=1e-2, factor_update_freq=2, decomp_update_freq=2,
                      weight_decay=1e-3, momentum=0.9, gamma=0.3)
    errs = []
    for s in range(1, 6):
        loss = F.cross_entropy(model(x), y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        for k, v in model.state_dict().items():
            errs.append((s, k, rel(v.detach().cpu().numpy(), g[f"{tag}_s{s}_{k}"])))
    stats = opt.get_timing_stats()
    opt.cleanup()
    return errs, stats


@pytest.mark.parametrize("tag", ["mlp", "conv"])
def test_classic_trajectory_matches_reference_cpu(tag):
    errs, stats = run_classic(tag, "cpu")
    assert max(e for _, _, e in errs) < 1e-5, max(errs, key=lambda t: t[2])
    assert stats["inversion"]["count"] == 3 and stats["total_step"]["count"] == 5


def test_hooks_capture_pause_and_gram_rows():
    from ifkfac_b200.classic_kfac import KFACHooks
    lin = nn.Linear(6, 3)
    h = KFACHooks(nn.Sequential(lin))
    h.enable()
    x = torch.randn(2, 5, 6)   # 3-D input: 10 token rows
    lin(x).sum().backward()
    A, G = h.get_factors()[lin]
    X = x.reshape(-1, 6)
    assert torch.allclose(A, X.t() @ X / 10, atol=1e-6)
    assert G.shape == (3, 3) and h.n_samples_accumulated() == 10
    h.pause()
    lin(x).sum().backward()
    assert h.n_samples_accumulated() == 10
    with h.capture():
        lin(x).sum().backward()
    assert h.n_samples_accumulated() == 20 and not h.is_enabled
    h.remove()
