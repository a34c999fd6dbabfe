"""DistributedIFKFAC on two GPUs (NCCL): batch-sharded TSQR reduced by the R-tree to
each layer's owner at each refresh, gradients averaged, each layer's solves and
update on its owner rank and broadcast.  Against IFKFAC on the full batch in one
process: the same factors (on the owners, the only ranks that hold them) and
trajectory up to the merge order of the rows (fp32 mode 1e-4; bf16 mode within its
2e-2 bound), and bit-identical parameters on every rank.
Skipped with fewer than two GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from ifkfac_b200 import _lib

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("prec,tol", [(_lib.PREC_FP32, 1e-4), (_lib.PREC_BF16, 2e-2)])
def test_distributed_optimizer_matches_single_process(prec, tol):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "dist_optimizer_worker.py"), str(prec)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    out = json.loads(line)
    assert out["same_on_ranks"] and out["owners"] == [0, 1] and out["factors_on_owners_only"]
    assert out["factor_rel_err"] < tol and out["weight_rel_err"] < tol, out
