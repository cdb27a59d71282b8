"""Worker for tests/test_multi_gpu.py (run under torchrun, one process per GPU):
a row-sharded chain whose phases feed each other through the in-kernel
exchange -- phase k's activation is the FULL output of phase k-1, half of
whose rows another GPU computed and stored over NVLink during the same launch.
Before every launch the full outputs are filled with NaN on every rank, so a
phase that read before the previous phase's rows had arrived would see NaN or
a stale value.  Every phase's full output is checked on every rank against
the float64 oracle applied to the previous phase's output."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "vram-compression_b200"))
import rans_b200 as rb       # noqa: E402
import rans_dist as rd       # noqa: E402
from oracle import rans_oracle as orc   # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rb.load()
    shapes = [(1024, 1536), (2048, 1024), (512, 2048), (1536, 512)]
    rng = np.random.default_rng(17)
    codes, shards, steps = [], [], []
    for i, (rows, cols) in enumerate(shapes):
        c = orc.synth_codes(rows, cols, 3.25, "laplace", seed=300 + i)
        step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32) if i == 0 else np.ones(cols, np.float32)
        enc = rb.encode(c, 8, 512)
        shard, _, _ = rb.shard_encoding(enc, rank, world)
        shards.append(rb.RansMatrix(shard, torch.from_numpy(step)))
        codes.append(c)
        steps.append(step)
    x0 = torch.from_numpy(rng.standard_normal(1536).astype(np.float32)).bfloat16().cuda()
    ch = rd.ShardedChain(shards, [r for r, _ in shapes], [x0, 0, 1, 2], [0, 1, 2, 3], timeout_ms=5000)
    worst = 0.0
    for it in range(20):
        ch.y_full.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        ch()
        ch.check()
        # the last phase's rows from the other rank are complete once that
        # rank's launch has ended too
        torch.cuda.synchronize()
        dist.barrier()
        xin = x0.float().cpu().numpy().astype(np.float64) * steps[0].astype(np.float64)
        for k in range(4):
            got = ch.full[k].cpu().numpy().astype(np.float64)
            if not np.all(np.isfinite(got)):
                raise AssertionError(f"iteration {it}: phase {k} read rows that had not arrived")
            ref = orc.gemv(codes[k], np.ones(codes[k].shape[1]), xin)
            err = orc.rel_l2(got, ref)
            worst = max(worst, err)
            if err > 1e-3:
                raise AssertionError(f"iteration {it}: phase {k} rel-L2 {err}")
            xin = got
        dist.barrier()
    t = torch.tensor([worst], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(f"chain feed ok: world {world}, worst rel-L2 {t.item():.2e}")
    ch.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
