"""Tests that need two or more GPUs of one node: one process per GPU through
torch.distributed.run (127.0.0.1 rendezvous). Skipped on a one-GPU box."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def test_sharded_lm_head_peer_exchange_matches_one_gpu():
    """Config 5 on every GPU of the box (up to 8): the vocab-sharded lm_head's
    greedy ids and top-50 with the peer-memory exchange (push over NVLink,
    epoch flags) and with the NCCL all-gather both equal one GPU's results on
    the whole vocabulary, over five calls and two batch shapes."""
    n = min(gpus(), 8)
    if n < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_DEBUG="WARN")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29517",
           os.path.join(HERE, "multigpu_lmhead.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    out = res.stdout + res.stderr
    assert res.returncode == 0, out[-4000:]
    assert out.count("OK rank") == n, out[-4000:]
