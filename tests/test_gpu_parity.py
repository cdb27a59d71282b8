"""GPU parity: librans_b200 against the oracle (and the reference's own outputs
recorded in tests/golden), through the C ABI.

Bars (from the reference's kernel/bench.py:38-66 and the task's north star):
  * decoded codes bit-exact (decode with step = 1 returns bf16(code) exactly);
  * decode to bf16 equals bf16(code * step) bit for bit (bench.py:49-51);
  * GEMV: relative L2 <= 1e-3 against float64 dequantise-then-matvec, and the
    reference's own max-abs-relative bound 1e-4 (bench.py:52-56);
  * int4 baseline: allclose(rtol=1e-4, atol=1e-3) (bench.py:65).
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, golden_cases, load_case
from oracle import rans_oracle as orc

pytestmark = pytest.mark.gpu

CASES = golden_cases()
IDS = [os.path.basename(p)[:-4] for p in CASES]
REL_L2 = 1e-3      # north-star GEMV tolerance
MAX_REL = 1e-4     # kernel/bench.py:55


@pytest.fixture(scope="module")
def torch(cuda_ok):
    import torch as t
    return t


@pytest.fixture(scope="module")
def rb():
    import rans_b200
    rans_b200.load()
    return rans_b200


def _y64(codes, step, x):
    return orc.gemv(codes, step.astype(np.float64), x.astype(np.float64))


def _check_y(y, yref):
    y = np.asarray(y, np.float64)
    assert orc.rel_l2(y, yref) <= REL_L2
    assert np.abs(y - yref).max() / max(np.abs(yref).max(), 1e-30) < MAX_REL


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_decode_bit_exact(torch, rb, path):
    codes, enc, step, x, y, _ = load_case(path)
    m = rb.RansMatrix(enc, torch.ones(codes.shape[1]))
    got = m.decode().float().cpu().numpy()
    assert np.array_equal(got.astype(np.int64), codes)
    m2 = rb.RansMatrix(enc, torch.from_numpy(step))
    dec = m2.decode().cpu()
    want = (torch.from_numpy(codes).float() * torch.from_numpy(step)).bfloat16()
    assert torch.equal(dec, want)


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_gemv_dropin(torch, rb, path):
    codes, enc, step, x, y, _ = load_case(path)
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    got = m.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    _check_y(got, y)
    # an explicit, dirty y buffer is zeroed by the wrapper when cols != C
    yb = torch.full((m.rows,), 7.0, device="cuda")
    got2 = m.gemv(torch.from_numpy(x).cuda(), yb).cpu().numpy()
    _check_y(got2, y)


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_gemv_bf16_fused_step(torch, rb, path):
    codes, enc, step, x, y, _ = load_case(path)
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    xb = torch.from_numpy(x).bfloat16()
    yref = _y64(codes, step, xb.float().numpy())
    got = m.gemv_bf16(xb.cuda(), torch.full((m.rows,), float("nan"), device="cuda")).cpu().numpy()
    _check_y(got, yref)


def test_step_launcher_matches_single(torch, rb):
    mats, xs, ys, refs = [], [], [], []
    for path in CASES:
        codes, enc, step, x, y, _ = load_case(path)
        if enc["R"] != 8:
            continue
        m = rb.RansMatrix(enc, torch.from_numpy(step))
        xb = torch.from_numpy(x).bfloat16().cuda()
        mats.append(m)
        xs.append(xb)
        ys.append(torch.full((m.rows,), float("nan"), device="cuda"))
        refs.append(_y64(codes, step, xb.float().cpu().numpy()))
    assert len(mats) >= 3
    step = rb.RansStep(mats, xs, ys)
    for _ in range(2):
        step()
        torch.cuda.synchronize()
        for yv, yr in zip(ys, refs):
            _check_y(yv.cpu().numpy(), yr)


@pytest.mark.parametrize("shape,R,C,dist,bits", [
    ((1536, 1536), 8, 512, "laplace", 3.25),
    ((8960, 1536), 8, 512, "gauss", 4.25),       # config 2 gate/up
    ((1536, 8960), 8, 640, "gauss", 4.25),       # config 2 down
    ((512, 2048), 16, 512, "laplace", 2.25),     # config 3, R=16
    ((256, 1024), 4, 1024, "laplace", 2.25),     # row mode, R=4
])
def test_large_against_c_oracle(torch, rb, shape, R, C, dist, bits):
    rows, cols = shape
    codes = orc.synth_codes(rows, cols, bits, dist, seed=rows + cols)
    rng = np.random.default_rng(rows)
    step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    enc = rb.encode(codes, R, C)
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    xb = torch.from_numpy(x).bfloat16()
    xs = xb.float().numpy().astype(np.float64) * step.astype(np.float64)
    yref = orc.c_decode_gemv(enc, xs, threads=8)
    _check_y(m.gemv_bf16(xb.cuda()).cpu().numpy(), yref)
    yref32 = orc.c_decode_gemv(enc, x.astype(np.float64) * step.astype(np.float32).astype(np.float64), threads=8)
    _check_y(m.gemv(torch.from_numpy(x).cuda()).cpu().numpy(), yref32)
    dec = m.decode().cpu()
    want = (torch.from_numpy(codes).float() * torch.from_numpy(step)).bfloat16()
    assert torch.equal(dec, want)


@pytest.mark.parametrize("kind", ["two", "extremes", "dominant"])
@pytest.mark.parametrize("R", [1, 8, 16])
def test_edge_distributions(torch, rb, kind, R):
    """Code distributions at the edges of the 12-bit table: two symbols only
    (one of them rare: long runs without a renormalisation word), the
    alphabet's extremes -128 and 127 only, and one dominant symbol with up to
    300 singletons (frequency 1 each).  Decode bit-exact against
    bf16(code * step); both GEMV entry points against float64."""
    rng = np.random.default_rng({"two": 1, "extremes": 2, "dominant": 3}[kind] * 100 + R)
    rows, cols, C = 16 * R, 1536, 512
    if kind == "two":
        codes = np.where(rng.random((rows, cols)) < 0.002, 5, -3)
    elif kind == "extremes":
        codes = np.where(rng.random((rows, cols)) < 0.5, -128, 127)
    else:
        codes = np.zeros((rows, cols), np.int64)
        idx = rng.choice(rows * cols, 300, replace=False)
        codes.flat[idx] = rng.choice(np.r_[-128:0, 1:128], 300)
    codes = codes.astype(np.int32)
    step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    enc = rb.encode(codes, R, C)
    ref = orc.encode(codes, R, C)
    assert np.array_equal(enc["words"], ref["words"]) and np.array_equal(enc["offs"], ref["offs"])
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    _check_y(m.gemv(torch.from_numpy(x).cuda()).cpu().numpy(), _y64(codes, step, x))
    xb = torch.from_numpy(x).bfloat16()
    _check_y(m.gemv_bf16(xb.cuda()).cpu().numpy(), _y64(codes, step, xb.float().numpy()))
    dec = m.decode().float().cpu().numpy()
    assert np.array_equal(dec, (torch.from_numpy(codes).float() * torch.from_numpy(step)).bfloat16().float().numpy())


def test_unstaged_fallback_high_entropy(torch, rb):
    """Spans larger than the shared-memory stage (8 bits/symbol, R=16, C=1024)
    take the global-memory path; results must not change."""
    rng = np.random.default_rng(3)
    codes = rng.integers(-128, 128, (64, 2048)).astype(np.int32)
    step = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    x = rng.standard_normal(2048).astype(np.float32)
    enc = rb.encode(codes, 16, 1024)
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    _check_y(m.gemv(torch.from_numpy(x).cuda()).cpu().numpy(), _y64(codes, step, x))
    xb = torch.from_numpy(x).bfloat16()
    _check_y(m.gemv_bf16(xb.cuda()).cpu().numpy(), _y64(codes, step, xb.float().numpy()))
    dec = m.decode().float().cpu().numpy()
    assert np.array_equal(dec, (torch.from_numpy(codes).float() * torch.from_numpy(step)).bfloat16().float().numpy())


def test_int4_baseline(torch, rb):
    """kernel/bench.py:59-66: int4 codes, default_rng(1), 256x1024."""
    codes = np.random.default_rng(1).integers(-8, 8, size=(256, 1024))
    g = torch.Generator().manual_seed(0)
    step = torch.rand(1024, generator=g) + 0.5
    m4 = rb.Int4Matrix(codes, step)
    x = torch.randn(1024, generator=g).cuda()
    y_ref = torch.from_numpy(codes).float().cuda() @ (x * step.cuda())
    assert torch.allclose(m4.gemv(x), y_ref, rtol=1e-4, atol=1e-3)
    for rows, cols in ((1536, 8960), (100, 64)):
        c = np.random.default_rng(rows).integers(-8, 8, size=(rows, cols))
        s = torch.rand(cols, generator=g) + 0.5
        xx = torch.randn(cols, generator=g).cuda()
        mm = rb.Int4Matrix(c, s)
        yr = torch.from_numpy(c).float().cuda() @ (xx * s.cuda())
        assert torch.allclose(mm.gemv(xx), yr, rtol=1e-4, atol=1e-3)


def test_reference_kernel_agrees(torch, rb):
    """The reference's own kernel, compiled unmodified for sm_100a into
    oracle/_ref, gives the same decode and (within fp32 order) the same GEMV."""
    ref_so = os.path.join(ROOT, "oracle", "_ref", "librans_ref.so")
    if not os.path.exists(ref_so):
        pytest.skip("oracle/_ref/librans_ref.so not built")
    ref = ctypes.CDLL(ref_so)
    for f in (ref.launch_rans_gemv, ref.launch_rans_decode):
        f.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
        f.restype = ctypes.c_int
    codes, enc, step, x, y, _ = load_case(os.path.join(GOLDEN, "edge_gauss425_256x1536_R8_C512.npz"))
    mine = rb.RansMatrix(enc, torch.from_numpy(step))
    theirs = rb.RansMatrix(enc, torch.from_numpy(step), lib=ref)
    assert torch.equal(mine.decode(), theirs.decode())
    xt = torch.from_numpy(x).cuda()
    a = mine.gemv(xt).cpu().numpy()
    b = theirs.gemv(xt).cpu().numpy()
    assert orc.rel_l2(a, b) < 1e-5


def test_chained_steps_read_previous_output(torch, rb):
    """Step kernels start early (programmatic dependent launch) but must read
    activations only after the previous kernel finished: launch B's input is
    launch A's output (fp32, already step-scaled), repeated back to back."""
    rng = np.random.default_rng(11)
    codes_a = orc.synth_codes(1024, 1536, 3.25, "laplace", seed=21)   # y_a has 1024 rows
    codes_b = orc.synth_codes(512, 1024, 4.25, "gauss", seed=22)      # consumes 1024 columns
    step_a = (0.01 * rng.uniform(0.5, 1.5, 1536)).astype(np.float32)
    ma = rb.RansMatrix(rb.encode(codes_a, 8, 512), torch.from_numpy(step_a))
    mb = rb.RansMatrix(rb.encode(codes_b, 8, 512), torch.ones(1024))
    xa = torch.from_numpy(rng.standard_normal(1536).astype(np.float32)).bfloat16().cuda()
    ya = torch.empty(1024, device="cuda")
    yb = torch.empty(512, device="cuda")
    sa = rb.RansStep([ma], [xa], [ya])
    sb = rb.RansStep([mb], [ya], [yb], prescaled_x=True)   # B reads ya as fp32, already scaled
    ya_ref = orc.gemv(codes_a, step_a.astype(np.float64), xa.float().cpu().numpy().astype(np.float64))
    for _ in range(20):
        ya.fill_(float("nan"))
        yb.fill_(float("nan"))
        sa()
        sb()
    torch.cuda.synchronize()
    _check_y(ya.cpu().numpy(), ya_ref)
    yb_ref = orc.gemv(codes_b, np.ones(1024), ya.cpu().numpy().astype(np.float64))
    _check_y(yb.cpu().numpy(), yb_ref)


def test_throughput_step_prescale_reads_fresh_activations(torch, rb):
    """A throughput plan (enough whole-row items, not split) first turns bf16
    x into x*step in its workspace with a small kernel, then decodes.  The
    activations are rewritten by an ordinary kernel before every launch; each
    launch must see the new values (the prescale waits for the previous
    kernel of the stream), and the result must match the float64 oracle."""
    mats, xs, ys, codes_l, steps = [], [], [], [], []
    encs = {}
    for seed in (31, 32):
        codes = orc.synth_codes(8960, 1536, 4.25, "gauss", seed=seed)
        encs[seed] = (codes, rb.encode(codes, 8, 512))
    for i in range(6):   # 6 x 1120 whole-row items: a multi-wave launch, so the plan prescales
        seed = 31 + i % 2
        codes, enc = encs[seed]
        step = (0.01 * np.random.default_rng(100 + i).uniform(0.5, 1.5, 1536)).astype(np.float32)
        mats.append(rb.RansMatrix(enc, torch.from_numpy(step)))
        xs.append(torch.empty(1536, device="cuda", dtype=torch.bfloat16))
        ys.append(torch.empty(8960, device="cuda"))
        codes_l.append(codes)
        steps.append(step)
    st = rb.RansStep(mats, xs, ys)
    g = torch.Generator(device="cuda").manual_seed(5)
    for it in range(6):
        srcs = [torch.randn(1536, device="cuda", generator=g) for _ in xs]
        for x, src in zip(xs, srcs):
            x.copy_(src.bfloat16())
        st()
    torch.cuda.synchronize()
    for x, y, codes, step in zip(xs, ys, codes_l, steps):
        _check_y(y.cpu().numpy(), _y64(codes, step, x.float().cpu().numpy()))


def test_medium_launch_segments_rows(torch, rb):
    """A launch of a few waves of whole-row items (8 down projections,
    1536 x 8960: 1536 row blocks of 7 two-tile passes) is cut into row
    segments that meet in the workspace; results must not change, including
    when the step is launched repeatedly (counters reset themselves)."""
    codes = orc.synth_codes(1536, 8960, 4.25, "gauss", seed=41)
    enc = rb.encode(codes, 8, 640)
    mats, xs, ys, steps = [], [], [], []
    for i in range(8):
        step = (0.01 * np.random.default_rng(200 + i).uniform(0.5, 1.5, 8960)).astype(np.float32)
        mats.append(rb.RansMatrix(enc, torch.from_numpy(step)))
        xs.append(torch.from_numpy(np.random.default_rng(300 + i).standard_normal(8960).astype(np.float32))
                  .bfloat16().cuda())
        ys.append(torch.full((1536,), float("nan"), device="cuda"))
        steps.append(step)
    st = rb.RansStep(mats, xs, ys)
    for _ in range(3):
        for y in ys:
            y.fill_(float("nan"))
        st()
    torch.cuda.synchronize()
    for x, y, step in zip(xs, ys, steps):
        _check_y(y.cpu().numpy(), _y64(codes, step, x.float().cpu().numpy()))


@pytest.mark.parametrize("rows,cols,R,C,bits", [
    (256, 8960, 8, 8960, 4.25),    # one tile of 71680 symbols per row block (C = cols)
    (64, 4096, 16, 4096, 2.25),    # R = 16, C = cols
    (512, 2048, 4, 2048, 5.0),     # R = 4, C = 2048
])
def test_tiles_larger_than_the_stage(torch, rb, rows, cols, R, C, bits):
    """Tiles whose words exceed the 8 KB per-warp stage decode through windows
    of each lane's stream: results match the oracle for the drop-in entry
    (buffer length unknown), the bf16 entry (length known), the step launcher
    and the decode to dense bf16."""
    codes = orc.synth_codes(rows, cols, bits, "gauss", seed=rows + C)
    rng = np.random.default_rng(cols)
    step = (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    enc = rb.encode(codes, R, C)
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    _check_y(m.gemv(torch.from_numpy(x).cuda()).cpu().numpy(), _y64(codes, step, x))
    xb = torch.from_numpy(x).bfloat16()
    yref = _y64(codes, step, xb.float().numpy())
    _check_y(m.gemv_bf16(xb.cuda()).cpu().numpy(), yref)
    y = torch.full((rows,), float("nan"), device="cuda")
    rb.RansStep([m], [xb.cuda()], [y])()
    torch.cuda.synchronize()
    _check_y(y.cpu().numpy(), yref)
    # decode to dense bf16 through the same windows, bit-exact
    want = (torch.from_numpy(codes).float() * torch.from_numpy(step)).bfloat16()
    assert torch.equal(m.decode().cpu(), want)
