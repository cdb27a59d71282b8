"""Row-sharded multi-GPU path on real GPUs (skipped with fewer than 2).

Runs bench.py under torchrun on 2 GPUs (2 layers of the Llama-3-70B-shaped
chain): its built-in checks must pass -- every rank's rows of the first and
last layer against the float64 oracle, and every rank holding identical full
outputs after the in-kernel exchange (each phase's rows stored into every
rank's buffer, then an in-kernel wait for every rank's arrival signal).
"""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_gpu_chain_exchange_checks(cuda_ok):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "bench.py"), "--gpus", "2", "--layers", "2", "--steps", "5", "--warmup", "3",
           "--no-cpu-baseline"]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=700)
    assert out.returncode == 0, out.stderr[-3000:]
    line = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])
    assert line["n_gpus"] == 2
    assert line["check"]["ok"], line["check"]
    assert line["check"]["exchange_identical_on_all_ranks"]


def test_two_gpu_chain_phases_feed_each_other(cuda_ok):
    """Phase k reads the full output of phase k-1 exchanged inside the same
    launch (tests/mgpu_chain_feed.py): every phase on every rank must match the
    oracle over 20 launches whose outputs are reset to NaN first."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "mgpu_chain_feed.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=400)
    assert out.returncode == 0, out.stderr[-3000:]
    assert "chain feed ok" in out.stdout
