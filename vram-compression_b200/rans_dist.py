"""Row-sharded multi-GPU decoder step (one process per GPU, torch.distributed).

Every projection's row blocks are split into one contiguous range per rank
(`shard_rows`, the same split as rans_b200.shard_encoding); because the streams
of consecutive row blocks are consecutive, a rank's shard is a slice of the
encoding, not a re-encoding.  Each rank decodes its rows of every projection
in one step launch, and the outputs are exchanged in one of two ways:

  fused  the step kernel's epilogue stores every output row into the FULL
         output buffer of every rank (torch symmetric memory, NVLink stores),
         then one cross-GPU barrier (bounded: it raises after `timeout_ms`);
  nccl   the step writes local rows, then one all-gather per call
         (`gather_rows`, any backend: NCCL on GPUs, gloo on CPU).

ShardedChain runs a dependency-ordered decoder step (rans_b200.RansChain)
the same way: one launch per rank, each phase's rows stored into every rank's
full outputs, and an in-kernel wait per phase for every rank's arrival signal
(bounded: a wait that runs out is reported by check()).

The reference has no multi-GPU path; this is the exchange step its survey
describes (one all-gather of y per projection), fused into the kernel.
"""
from __future__ import annotations

import numpy as np

import rans_b200 as rb


def shard_rows(rows: int, R: int, rank: int, world: int):
    """(first row, row count) of `rank`'s contiguous row-block range."""
    if rows % R:
        raise ValueError("rows must be a multiple of R")
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    nrb = rows // R
    rb0, rb1 = nrb * rank // world, nrb * (rank + 1) // world
    return rb0 * R, (rb1 - rb0) * R


class ShardLayout:
    """Where every projection's shard rows live in the concatenated full
    outputs: projection i occupies [F[i], F[i] + rows[i]) of the full buffer
    and rank r's rows of it start at F[i] + row0[i][r]."""

    def __init__(self, rows, R: int, world: int):
        self.rows = [int(r) for r in rows]
        self.R, self.world = R, world
        self.F = np.concatenate([[0], np.cumsum(self.rows)[:-1]]).astype(np.int64)
        self.total = int(sum(self.rows))
        self.row0 = [[shard_rows(r, R, k, world)[0] for k in range(world)] for r in self.rows]
        self.nrows = [[shard_rows(r, R, k, world)[1] for k in range(world)] for r in self.rows]

    def local_slices(self, rank: int):
        """(start, stop) of rank's rows of every projection in the full buffer."""
        return [(int(self.F[i]) + self.row0[i][rank], int(self.F[i]) + self.row0[i][rank] + self.nrows[i][rank])
                for i in range(len(self.rows))]

    def peer_addresses(self, buffer_ptrs, rank: int, elem_bytes: int = 4):
        """Per projection, the address of rank's first shard row inside every
        rank's full buffer (buffer_ptrs[p] = base address of rank p's buffer as
        seen from this GPU)."""
        if len(buffer_ptrs) != self.world:
            raise ValueError("one buffer pointer per rank")
        return [[int(buffer_ptrs[p]) + elem_bytes * (int(self.F[i]) + self.row0[i][rank])
                 for p in range(self.world)] for i in range(len(self.rows))]


def gather_rows(local, counts, group=None):
    """All-gather row shards of different lengths (rank order) into the full
    vector: pad to the longest shard, all_gather, trim.  Any backend."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if len(counts) != world:
        raise ValueError("one row count per rank")
    mx = max(int(c) for c in counts)
    buf = torch.zeros(mx, dtype=local.dtype, device=local.device)
    buf[: local.numel()] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p[: int(c)] for p, c in zip(parts, counts)])


def regroup_rank_major(gathered, layout: ShardLayout):
    """Rank-major gathered rows (rank 0's rows of projections 0..n-1, then
    rank 1's, ...) -> the full output of every projection."""
    import torch
    out = [torch.empty(r, dtype=gathered.dtype, device=gathered.device) for r in layout.rows]
    pos = 0
    for r in range(layout.world):
        for i in range(len(out)):
            n, a = layout.nrows[i][r], layout.row0[i][r]
            out[i][a:a + n].copy_(gathered[pos:pos + n])
            pos += n
    if pos != gathered.numel():
        raise ValueError("gathered rows do not match the layout")
    return out


class ShardedStep:
    """This rank's share of a decoder step whose projections are row-sharded
    over the ranks of the default process group.

    mats: this rank's row shards (RansMatrix, in projection order, e.g. from
    rans_b200.shard_encoding); full_rows: every projection's full row count;
    xs: this rank's activations (bf16, all columns).  After a call, `full[i]`
    is projection i's complete output on this rank (fused exchange), or
    `full_outputs()` assembles it (nccl exchange, one all-gather per call).
    """

    def __init__(self, mats, full_rows, xs, exchange: str = "fused", timeout_ms: int = 60000, lib=None):
        import torch
        import torch.distributed as dist
        if exchange not in ("fused", "nccl"):
            raise ValueError("exchange must be 'fused' or 'nccl'")
        if len(mats) != len(full_rows) or len(xs) != len(mats):
            raise ValueError("one shard, one full row count and one activation per projection")
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        R = mats[0].R
        self.layout = ShardLayout(full_rows, R, self.world)
        for i, m in enumerate(mats):
            if m.rows != self.layout.nrows[i][self.rank]:
                raise ValueError(f"projection {i}: shard has {m.rows} rows, "
                                 f"rank {self.rank} owns {self.layout.nrows[i][self.rank]}")
        dev = mats[0].device
        self.exchange, self.timeout_ms = exchange, timeout_ms
        self.mats = list(mats)
        sl = self.layout.local_slices(self.rank)
        self.hdl = None
        if exchange == "fused":
            import torch.distributed._symmetric_memory as symm_mem
            self.y_full = symm_mem.empty(self.layout.total, dtype=torch.float32, device=dev)
            self.y_full.zero_()
            try:
                self.hdl = symm_mem.rendezvous(self.y_full, dist.group.WORLD)
            except Exception:
                symm_mem.enable_symm_mem_for_group(dist.group.WORLD.group_name)
                self.hdl = symm_mem.rendezvous(self.y_full, dist.group.WORLD)
            peers = self.layout.peer_addresses([int(p) for p in self.hdl.buffer_ptrs], self.rank)
            ys = [self.y_full[a:b] for a, b in sl]
            self.step = rb.RansStep(self.mats, xs, ys, lib=lib, peers=peers)
            self.full = [self.y_full[int(self.layout.F[i]):int(self.layout.F[i]) + self.layout.rows[i]]
                         for i in range(len(mats))]
        else:
            n_local = sum(b - a for a, b in sl)
            self.y_local = torch.zeros(n_local, device=dev)
            offs = np.concatenate([[0], np.cumsum([b - a for a, b in sl])]).astype(np.int64)
            ys = [self.y_local[int(offs[i]):int(offs[i + 1])] for i in range(len(sl))]
            self.step = rb.RansStep(self.mats, xs, ys, lib=lib)
            # rank r's local buffer holds its rows of every projection in order
            self._counts = [sum(self.layout.nrows[i][r] for i in range(len(sl))) for r in range(self.world)]
            self.gathered = None
            self.full = None

    @property
    def kernels(self) -> int:
        return self.step.kernels

    def __call__(self):
        if self.exchange == "fused":
            # The kernel stores into every rank's full outputs: first make sure
            # no rank still reads the previous call's result (back-to-back
            # calls would otherwise overwrite it under a slower rank).
            self.hdl.barrier(channel=1, timeout_ms=self.timeout_ms)
        self.step()
        if self.exchange == "fused":
            # every rank's rows are in every rank's buffer once all ranks have
            # passed this barrier (it raises after timeout_ms)
            self.hdl.barrier(channel=0, timeout_ms=self.timeout_ms)
        else:
            self.gathered = gather_rows(self.y_local, self._counts)
        return self.full

    def full_outputs(self):
        """Complete outputs of every projection (a copy for the nccl exchange)."""
        if self.exchange == "fused":
            return self.full
        return regroup_rank_major(self.gathered, self.layout)

    def close(self):
        """Drop the plan and the symmetric-memory handle before the process
        group is destroyed."""
        self.step = None
        self.hdl = None


def _symm_rendezvous(t):
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem
    try:
        return symm_mem.rendezvous(t, dist.group.WORLD)
    except Exception:
        symm_mem.enable_symm_mem_for_group(dist.group.WORLD.group_name)
        return symm_mem.rendezvous(t, dist.group.WORLD)


class ShardedChain:
    """This rank's share of a dependency-ordered decoder step (phases) whose
    projections are row-sharded over the ranks of the default process group.

    mats / full_rows / xs as for ShardedStep, except that xs[i] may be an int
    j: projection i then reads the FULL output of projection j (fp32, already
    multiplied by the step: the pre-scaled convention), produced by an earlier
    phase of the same launch and exchanged by the kernel; phases[i] is
    projection i's phase.  One call is one kernel launch on this rank: phase p+1 starts once
    every rank has stored its rows of phase p into every rank's `y_full`
    (symmetric memory) and signalled it.  `full[i]` is projection i's complete
    output on this rank once every rank's launch has ended (nothing inside the
    kernel waits for the last phase: synchronise and pass a barrier before
    reading it on the host).  Every rank must call the
    same number of times; check() synchronises and raises
    rans_b200.ChainTimeout if a wait ran out (then build the chain again on
    every rank).
    """

    def __init__(self, mats, full_rows, xs, phases, timeout_ms: int = 5000, lib=None, prescaled_x=False):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        if len(mats) != len(full_rows) or len(xs) != len(mats) or len(phases) != len(mats):
            raise ValueError("one shard, one full row count, one activation and one phase per projection")
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        R = mats[0].R
        self.layout = ShardLayout(full_rows, R, self.world)
        for i, m in enumerate(mats):
            if m.rows != self.layout.nrows[i][self.rank]:
                raise ValueError(f"projection {i}: shard has {m.rows} rows, "
                                 f"rank {self.rank} owns {self.layout.nrows[i][self.rank]}")
        dev = mats[0].device
        nphases = max(int(p) for p in phases) + 1
        self.y_full = symm_mem.empty(self.layout.total, dtype=torch.float32, device=dev)
        self.y_full.zero_()
        self.hdl = _symm_rendezvous(self.y_full)
        # one more than the caller's phases: the chain may add an activation
        # prescale phase in front
        self.arrive = symm_mem.empty(max(nphases + 1, 4), dtype=torch.int32, device=dev)
        self.arrive.zero_()
        self.hdl_arrive = _symm_rendezvous(self.arrive)
        peers = self.layout.peer_addresses([int(p) for p in self.hdl.buffer_ptrs], self.rank)
        arrive_peer = [int(p) for p in self.hdl_arrive.buffer_ptrs]
        sl = self.layout.local_slices(self.rank)
        ys = [self.y_full[a:b] for a, b in sl]
        self.full = [self.y_full[int(self.layout.F[i]):int(self.layout.F[i]) + self.layout.rows[i]]
                     for i in range(len(mats))]
        feeds = [isinstance(x, int) for x in xs]
        xs = [self.full[x] if f else x for x, f in zip(xs, feeds)]
        pre = list(prescaled_x) if isinstance(prescaled_x, (list, tuple)) else [bool(prescaled_x)] * len(mats)
        pre = [p or f for p, f in zip(pre, feeds)]
        torch.cuda.synchronize()
        self.chain = rb.RansChain(mats, xs, ys, phases, lib=lib, prescaled_x=pre, timeout_ms=timeout_ms,
                                  sync=(self.world, self.rank, self.arrive.data_ptr(), arrive_peer, peers))
        # every rank has zeroed its arrival counters before any rank launches
        dist.barrier()
        self.kernels = 1

    def __call__(self):
        self.chain()
        return self.full

    def check(self):
        self.chain.check()

    def close(self):
        """Drop the plan and the symmetric-memory handles before the process
        group is destroyed."""
        self.chain = None
        self.hdl = None
        self.hdl_arrive = None
