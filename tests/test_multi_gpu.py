"""Row-sharded multi-GPU path on real GPUs (skipped with fewer than 2).

Runs bench.py under torchrun on 2 GPUs with --check: the fused exchange
(kernel epilogue storing every output row into all ranks' buffers, then one
cross-GPU barrier) must equal an NCCL all-gather of the same shard outputs
bit for bit.
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


def test_two_gpu_fused_exchange_matches_nccl(cuda_ok):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "bench.py"), "--gpus", "2", "--layers", "2", "--steps", "5", "--warmup", "3",
           "--check", "--no-cpu-baseline"]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=700)
    assert out.returncode == 0, out.stderr[-3000:]
    line = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])
    assert line["n_gpus"] == 2
    assert line["exchange"]["check"]["ok"], line["exchange"]
