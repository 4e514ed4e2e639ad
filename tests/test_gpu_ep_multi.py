"""Quantized peer-memory expert parallelism across real GPUs (CUDA IPC
between processes): each rank's output against the full single-GPU layer.
Needs at least 2 visible GPUs; runs the ranks under torchrun."""
import json
import os
import socket
import subprocess
import sys

import pytest

from moe_testutil import MAX_ABS_TOL, REL_L2_TOL

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,n,E,k", [(2, 300, 8, 4), (2, 64, 4, 2), (4, 300, 8, 4), (4, 256, 128, 4), (8, 256, 32, 4)])
def test_quantized_peer_ep_across_gpus(world, n, E, k):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "ep_multi_worker.py"), str(n), str(E), str(k)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("[")][-1]
    for rk in json.loads(line):
        assert rk["err"] == 0, rk
        for max_abs, rel in rk["errors"]:
            assert max_abs <= MAX_ABS_TOL and rel <= REL_L2_TOL, rk
