"""Row-block sharding of an encoding across ranks (the multi-GPU layout), on
CPU with gloo, world_size 2: each rank's shard is a valid standalone encoding
of its rows, and all-gathering the per-rank outputs reproduces the unsharded
result (the exchange step of the sharded path)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    import rans_b200 as rb
    from oracle import rans_oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ok = True
        for (rows, cols, R, C, seed) in [(96, 1024, 8, 512, 1), (64, 640, 16, 640, 2), (40, 256, 4, 128, 3)]:
            codes = orc.synth_codes(rows, cols, 3.25, "laplace", seed=seed)
            enc = orc.encode(codes, R, C)
            shard, row0, nrows = rb.shard_encoding(enc, rank, world)
            ok &= np.array_equal(orc.c_decode_codes(shard), codes[row0:row0 + nrows])
            ok &= int(shard["words"].size) % 1 == 0 and len(shard["offs"]) == nrows * cols * 32 // (R * C)
            xs = np.random.default_rng(seed).standard_normal(cols)
            y_local = torch.from_numpy(orc.c_decode_gemv(shard, xs))
            # ranks hold different row counts: pad to the largest shard, gather, trim
            n = torch.tensor([nrows])
            sizes = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
            dist.all_gather(sizes, n)
            mx = int(max(s.item() for s in sizes))
            buf = torch.zeros(mx, dtype=torch.float64)
            buf[:nrows] = y_local
            parts = [torch.zeros(mx, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(parts, buf)
            y = torch.cat([p[: int(s.item())] for p, s in zip(parts, sizes)]).numpy()
            ok &= np.allclose(y, orc.gemv(codes, np.ones(cols), xs), rtol=1e-12, atol=1e-9)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_row_shards_gather_to_full_result():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def test_shard_edges_single_rank_is_identity():
    import rans_b200 as rb
    from oracle import rans_oracle as orc
    codes = orc.synth_codes(32, 256, 3.0, "laplace", seed=5)
    enc = orc.encode(codes, 8, 128)
    shard, row0, nrows = rb.shard_encoding(enc, 0, 1)
    assert (row0, nrows) == (0, 32)
    assert np.array_equal(shard["words"][: enc["words"].size], enc["words"])
    assert np.array_equal(orc.c_decode_codes(shard), codes)
