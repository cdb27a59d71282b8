"""Host logic of the row-sharded multi-GPU step (rans_dist) on CPU: the shard
split, the output layout and peer addresses, the variable-size all-gather on
gloo ranks, and failure detection when a rank dies (host-side fault
injection: the rank exits, no GPU is involved)."""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, ROOT
from oracle import rans_oracle as orc
import rans_b200 as rb
import rans_dist as rd


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_rows_matches_shard_encoding(world):
    codes = orc.synth_codes(200, 256, 3.0, "laplace", seed=world)
    enc = orc.encode(codes, 8, 128)
    covered = []
    for r in range(world):
        _, row0, nrows = rb.shard_encoding(enc, r, world)
        assert rd.shard_rows(200, 8, r, world) == (row0, nrows)
        covered.append((row0, row0 + nrows))
    assert covered[0][0] == 0 and covered[-1][1] == 200
    assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))
    with pytest.raises(ValueError):
        rd.shard_rows(201, 8, 0, world)
    with pytest.raises(ValueError):
        rd.shard_rows(200, 8, world, world)


def test_layout_partitions_the_full_outputs():
    rows = [1536, 256, 256, 1536, 8960, 8960, 1536]
    for world in (1, 2, 4, 8):
        L = rd.ShardLayout(rows, 8, world)
        assert L.total == sum(rows)
        mark = np.zeros(L.total, np.int32)
        for r in range(world):
            for a, b in L.local_slices(r):
                mark[a:b] += 1
        assert np.all(mark == 1)
        ptrs = [1 << 40 | (p << 32) for p in range(world)]
        for r in range(world):
            addrs = L.peer_addresses(ptrs, r)
            for i, (a, _) in enumerate(L.local_slices(r)):
                assert addrs[i] == [ptrs[p] + 4 * a for p in range(world)]
        with pytest.raises(ValueError):
            L.peer_addresses(ptrs[:-1] if world > 1 else ptrs + ptrs, 0)


def test_regroup_rank_major():
    rows = [48, 16, 32]
    L = rd.ShardLayout(rows, 8, 3)
    full = [torch.arange(r, dtype=torch.float32) + 1000 * i for i, r in enumerate(rows)]
    parts = []
    for r in range(3):
        for i in range(len(rows)):
            a, n = L.row0[i][r], L.nrows[i][r]
            parts.append(full[i][a:a + n])
    got = rd.regroup_rank_major(torch.cat(parts), L)
    assert all(torch.equal(g, f) for g, f in zip(got, full))
    with pytest.raises(ValueError):
        rd.regroup_rank_major(torch.zeros(sum(rows) + 1), L)


def _gather_worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    import rans_dist as rd
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        counts = [5, 3, 0][:world]
        local = torch.arange(counts[rank], dtype=torch.float64) + 100 * rank
        got = rd.gather_rows(local, counts)
        want = torch.cat([torch.arange(c, dtype=torch.float64) + 100 * r for r, c in enumerate(counts)])
        q.put((rank, bool(torch.equal(got, want))))
    finally:
        dist.destroy_process_group()


def test_gather_rows_variable_sizes_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True, 2: True}


def _dying_worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    import rans_dist as rd
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # fault injection: this rank dies between steps, before the exchange
        q.put((rank, "exited"))
        q.close()
        q.join_thread()    # flush the message before the hard exit
        os._exit(0)
    t0 = time.time()
    try:
        rd.gather_rows(torch.ones(4, dtype=torch.float64), [4, 4])
        q.put((rank, "no error"))
    except Exception as e:   # the surviving rank must fail, not hang
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_dead_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "exited"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 60
