"""The chain launcher (rans_gemv_chain_*): a decoder step as a chain of
dependent phases from one persistent grid, through the C ABI.

  * a 2-layer Qwen2.5-1.5B-shaped step (4 phases per layer) gives the
    outputs of one step launch per phase (the planner gives each phase the
    decomposition of a launch of its own, up to half-size items in the last
    wave of a multi-wave phase: equal within fp32 summation order) and matches
    the float64 oracle;
  * phases that really feed each other (phase p+1's activation is phase p's
    output) read the finished output in every one of 20 back-to-back launches;
  * a dependency that never arrives (a second rank that does not exist, on
    one GPU) makes the bounded wait run out: the status comes back, the
    context stays usable and the status clears once read;
  * every tile height R, and random chains of odd shapes and phase groupings.
"""
import numpy as np
import pytest

from oracle import rans_oracle as orc

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3      # north-star GEMV tolerance
MAX_REL = 1e-4     # kernel/bench.py:55

QWEN15B = [("q", 1536, 1536), ("k", 256, 1536), ("v", 256, 1536), ("o", 1536, 1536),
           ("gate", 8960, 1536), ("up", 8960, 1536), ("down", 1536, 8960)]
PHASE = {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3}


@pytest.fixture(scope="module")
def torch(cuda_ok):
    import torch as t
    return t


@pytest.fixture(scope="module")
def rb():
    import rans_b200
    rans_b200.load()
    return rans_b200


def _check_y(y, yref):
    y = np.asarray(y, np.float64)
    assert orc.rel_l2(y, yref) <= REL_L2
    assert np.abs(y - yref).max() / max(np.abs(yref).max(), 1e-30) < MAX_REL


def _c_tile(cols):
    return 512 if cols % 512 == 0 else 640


def test_chain_matches_one_launch_per_phase(torch, rb):
    layers = 2
    encs = {}
    mats, xs, phases, meta = [], [], [], []
    for li in range(layers):
        for pi, (name, rows, cols) in enumerate(QWEN15B):
            if pi not in encs:
                codes = orc.synth_codes(rows, cols, 4.25, "gauss", seed=50 + pi)
                encs[pi] = (codes, rb.encode(codes, 8, _c_tile(cols)))
            codes, enc = encs[pi]
            step = (0.01 * np.random.default_rng(1000 * li + pi).uniform(0.5, 1.5, cols)).astype(np.float32)
            mats.append(rb.RansMatrix(enc, torch.from_numpy(step)))
            xs.append(torch.randn(cols, generator=torch.Generator().manual_seed(77 + 10 * li + pi)).bfloat16().cuda())
            phases.append(4 * li + PHASE[name])
            meta.append((codes, step))
    ys_chain = [torch.full((m.rows,), float("nan"), device="cuda") for m in mats]
    chain = rb.RansChain(mats, xs, ys_chain, phases, timeout_ms=2000)
    ys_step = [torch.full((m.rows,), float("nan"), device="cuda") for m in mats]
    per_phase = []
    for p in sorted(set(phases)):
        idx = [i for i, q in enumerate(phases) if q == p]
        per_phase.append(rb.RansStep([mats[i] for i in idx], [xs[i] for i in idx], [ys_step[i] for i in idx]))
    for _ in range(3):          # repeated launches: the queue and counters reset themselves
        for y in ys_chain:
            y.fill_(float("nan"))
        chain()
        for st in per_phase:
            st()
    chain.check()
    torch.cuda.synchronize()
    for a, b in zip(ys_chain, ys_step):
        # same decomposition except the chain's half-size items in the last
        # wave of a multi-wave phase: equal up to fp32 summation order
        assert float((a - b).norm() / b.norm()) <= 1e-6
    for y, x, (codes, step) in zip(ys_chain, xs, meta):
        _check_y(y.cpu().numpy(), orc.gemv(codes, step.astype(np.float64), x.float().cpu().numpy().astype(np.float64)))


def test_chain_phases_feed_each_other(torch, rb):
    """x of phase p+1 is the fp32 output of phase p (already scaled: the
    matrices of phases 1..3 carry unit steps)."""
    shapes = [(1024, 1536), (2048, 1024), (512, 2048), (1536, 512)]
    rng = np.random.default_rng(5)
    codes_l, mats = [], []
    for i, (rows, cols) in enumerate(shapes):
        codes = orc.synth_codes(rows, cols, 3.25, "laplace", seed=90 + i)
        step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32) if i == 0 else np.ones(cols, np.float32)
        mats.append(rb.RansMatrix(rb.encode(codes, 8, 512), torch.from_numpy(step)))
        codes_l.append((codes, step))
    x0 = torch.from_numpy(rng.standard_normal(1536).astype(np.float32)).bfloat16().cuda()
    ys = [torch.empty(r, device="cuda") for r, _ in shapes]
    xs = [x0] + ys[:-1]
    chain = rb.RansChain(mats, xs, ys, [0, 1, 2, 3], prescaled_x=[False, True, True, True])
    for _ in range(20):
        for y in ys:
            y.fill_(float("nan"))
        chain()
    chain.check()
    torch.cuda.synchronize()
    xin = x0.float().cpu().numpy().astype(np.float64)
    for i, ((codes, step), y) in enumerate(zip(codes_l, ys)):
        got = y.cpu().numpy()
        _check_y(got, orc.gemv(codes, step.astype(np.float64), xin))
        xin = got.astype(np.float64)      # the next phase consumed exactly this output


def test_chain_wait_that_never_ends_reports_and_recovers(torch, rb):
    """Two 'ranks' on one GPU, the second never launches: phase 1 waits for an
    arrival that never comes, the wait runs out after the plan's timeout and
    the status says which phase; the GPU stays usable."""
    codes = orc.synth_codes(512, 1536, 3.25, "laplace", seed=12)
    step = (0.01 * np.random.default_rng(12).uniform(0.5, 1.5, 1536)).astype(np.float32)
    m = rb.RansMatrix(rb.encode(codes, 8, 512), torch.from_numpy(step))
    x = torch.randn(1536, generator=torch.Generator().manual_seed(3)).bfloat16().cuda()
    ys = [torch.empty(512, device="cuda") for _ in range(2)]
    dummy = [torch.zeros(512, device="cuda") for _ in range(2)]   # 'rank 1' output buffers
    arrive = torch.zeros(4, dtype=torch.int32, device="cuda")
    arrive_other = torch.zeros(4, dtype=torch.int32, device="cuda")  # nobody waits here
    peers = [[ys[i].data_ptr(), dummy[i].data_ptr()] for i in range(2)]
    sync = (2, 0, arrive.data_ptr(), [arrive.data_ptr(), arrive_other.data_ptr()], peers)
    xs = x.float() * torch.from_numpy(step).cuda()          # fp32 x*step: no prescale phase in front
    chain = rb.RansChain([m, m], [xs, xs], ys, [0, 1], timeout_ms=200, sync=sync, prescaled_x=True)
    chain()
    with pytest.raises(rb.ChainTimeout) as e:
        chain.check()
    assert e.value.phase == 0
    chain.check()                      # read once, then clear
    # the context is fine: an ordinary launch still works
    y = m.gemv_bf16(x)
    torch.cuda.synchronize()
    _check_y(y.cpu().numpy(), orc.gemv(codes, step.astype(np.float64), x.float().cpu().numpy().astype(np.float64)))


@pytest.mark.parametrize("R", [1, 2, 4, 16])
def test_chain_every_tile_height(torch, rb, R):
    """The chain launcher at every R the format allows: two latency-bound
    phases and a multi-wave one, the last feeding on the second's output."""
    rng = np.random.default_rng(40 + R)
    shapes = [(256, 1024), (512, 1024), (256 * 40, 512)]   # third: x = phase-1 output (512 rows)
    mats, codes_l, steps = [], [], []
    for i, (rows, cols) in enumerate(shapes):
        c = orc.synth_codes(rows, cols, 3.25, "laplace", seed=70 + 3 * R + i)
        step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32) if i < 2 else np.ones(cols, np.float32)
        mats.append(rb.RansMatrix(rb.encode(c, R, 512), torch.from_numpy(step)))
        codes_l.append(c)
        steps.append(step)
    x0 = torch.from_numpy(rng.standard_normal(1024).astype(np.float32)).bfloat16().cuda()
    ys = [torch.full((r,), float("nan"), device="cuda") for r, _ in shapes]
    ch = rb.RansChain(mats, [x0, x0, ys[1]], ys, [0, 1, 2], prescaled_x=[False, False, True])
    for _ in range(3):
        for y in ys:
            y.fill_(float("nan"))
        ch()
    ch.check()
    torch.cuda.synchronize()
    xb = x0.float().cpu().numpy().astype(np.float64)
    for k in range(2):
        _check_y(ys[k].cpu().numpy(), orc.gemv(codes_l[k], steps[k].astype(np.float64), xb))
    _check_y(ys[2].cpu().numpy(), orc.gemv(codes_l[2], np.ones(512), ys[1].cpu().numpy().astype(np.float64)))


@pytest.mark.parametrize("seed", range(6))
def test_random_chains(torch, rb, seed):
    """Random chains through the kernel (the planner's side of the same cases
    is checked without a GPU in tests/test_host.py): tile heights R 1-16, tile
    widths 64-640 columns, 1-7 column tiles, 1-80 row blocks, 1.25-6 bits
    per weight, random phase groupings, bf16 and prescaled fp32 activations
    mixed; every output of two back-to-back launches against float64."""
    rng = np.random.default_rng(900 + seed)
    R = (1, 2, 4, 8, 16, 8)[seed]
    n = int(rng.integers(3, 8))
    raw = rng.integers(0, n, n)
    used = sorted(set(raw.tolist()))
    phases = [used.index(v) for v in raw.tolist()]
    mats, codes_l, steps, xs, xref, pre = [], [], [], [], [], []
    for i in range(n):
        C = int(rng.choice([64, 256, 512, 640]))
        rows, cols = R * int(rng.integers(1, 81)), C * int(rng.integers(1, 8))
        bits = float(rng.choice([1.25, 2.25, 3.25, 4.25, 6.0]))
        codes = orc.synth_codes(rows, cols, bits, str(rng.choice(["laplace", "gauss"])), seed=1000 * seed + i)
        step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)
        x = rng.standard_normal(cols).astype(np.float32)
        mats.append(rb.RansMatrix(rb.encode(codes, R, C), torch.from_numpy(step)))
        codes_l.append(codes)
        if rng.random() < 0.5:                                   # bf16 x, step applied in the kernel
            xb = torch.from_numpy(x).bfloat16()
            xs.append(xb.cuda())
            xref.append(xb.float().numpy().astype(np.float64) * step.astype(np.float64))
            pre.append(False)
        else:                                                    # fp32 x already times the step
            xp = (torch.from_numpy(x) * torch.from_numpy(step)).float()
            xs.append(xp.cuda())
            xref.append(xp.numpy().astype(np.float64))
            pre.append(True)
    ys = [torch.empty(m.rows, device="cuda") for m in mats]
    ch = rb.RansChain(mats, xs, ys, phases, prescaled_x=pre)
    for _ in range(2):
        for y in ys:
            y.fill_(float("nan"))
        ch()
    ch.check()
    torch.cuda.synchronize()
    for i in range(n):
        _check_y(ys[i].cpu().numpy(), orc.gemv(codes_l[i], np.ones(codes_l[i].shape[1]), xref[i]))
