"""Every shape the benchmark times, against the CPU oracle, through the C ABI.

  * BASELINE config 4 (Qwen2.5-32B shapes, Gaussian codes at 3.25 b) and
    config 5 (Llama-3-70B shapes, Laplacian codes at 2.25 b with log-normal
    steps): the single-matrix bf16 entry, the drop-in entry (fp32 pre-scaled
    x), the step launcher and the chain launcher give y within rel-L2 1e-3 and
    max-abs-relative 1e-4 of the float64 decode+dot of the same encoding, and
    the decode to dense bf16 is bit-exact;
  * a whole 28-layer Qwen2.5-1.5B step (196 matrices, the plan bench.py's
    config 2 times: k/v with 256 rows beside gate/up with 8960, prescaled
    activations, chunk ordering) through one step launch and through the chain
    (112 dependent phases): every output against the oracle.
"""
import os

import numpy as np
import pytest

from oracle import rans_oracle as orc

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3      # north-star GEMV tolerance
MAX_REL = 1e-4     # kernel/bench.py:55
THREADS = max(1, len(os.sched_getaffinity(0)))


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


def _codes(torch, rows, cols, dist, bits, seed):
    """Codes of the benchmark's distribution (scale bisected as kernel/bench.py:29-33),
    drawn on the GPU for speed."""
    rng = np.random.default_rng(12345)
    w = rng.laplace(size=(256, 1536)) if dist == "laplace" else rng.standard_normal((256, 1536))
    lo, hi = -12.0, 6.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if orc.entropy_bits(np.round(w / np.exp(mid))) > bits:
            lo = mid
        else:
            hi = mid
    scale = float(np.exp(0.5 * (lo + hi)))
    g = torch.Generator(device="cuda").manual_seed(seed)
    if dist == "laplace":
        u = torch.rand(rows, cols, generator=g, device="cuda") - 0.5
        v = -torch.sign(u) * torch.log1p(-2 * u.abs())
    else:
        v = torch.randn(rows, cols, generator=g, device="cuda")
    return torch.clamp(torch.round(v / scale), -127, 127).to(torch.int8)


def _step(cols, dist, seed):
    rng = np.random.default_rng(seed)
    if dist == "laplace":
        return (0.01 * np.exp(rng.normal(0.0, 0.5, cols))).astype(np.float32)
    return (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)


@pytest.mark.parametrize("rows,cols,dist,bits", [
    (5120, 5120, "gauss", 3.25), (1024, 5120, "gauss", 3.25),          # config 4: q/o, k/v
    (27648, 5120, "gauss", 3.25), (5120, 27648, "gauss", 3.25),        # config 4: gate/up, down
    (8192, 8192, "laplace", 2.25), (1024, 8192, "laplace", 2.25),      # config 5: q/o, k/v
    (28672, 8192, "laplace", 2.25), (8192, 28672, "laplace", 2.25),    # config 5: gate/up, down
])
def test_benchmark_shapes_against_c_oracle(torch, rb, rows, cols, dist, bits):
    codes_d = _codes(torch, rows, cols, dist, bits, seed=rows + 7 * cols)
    enc = rb.encode(codes_d.cpu().numpy(), 8, 512, nthreads=THREADS)
    step = _step(cols, dist, rows)
    m = rb.RansMatrix(enc, torch.from_numpy(step))
    xb = torch.randn(cols, generator=torch.Generator().manual_seed(cols)).bfloat16()
    xs = xb.float().numpy().astype(np.float64) * step.astype(np.float64)
    yref = orc.c_decode_gemv(enc, xs, threads=THREADS)
    xd = xb.cuda()
    _check_y(m.gemv_bf16(xd).cpu().numpy(), yref)
    y1 = torch.full((rows,), float("nan"), device="cuda")
    rb.RansStep([m], [xd], [y1])()
    y2 = torch.full((rows,), float("nan"), device="cuda")
    ch = rb.RansChain([m], [xd], [y2], [0])
    ch()
    ch.check()
    _check_y(y1.cpu().numpy(), yref)
    _check_y(y2.cpu().numpy(), yref)
    # drop-in entry: fp32 x already multiplied by the step (kernel/rans.py:141)
    xf = torch.randn(cols, generator=torch.Generator().manual_seed(cols + 1))
    yref32 = orc.c_decode_gemv(enc, xf.numpy().astype(np.float64) * step.astype(np.float32).astype(np.float64),
                               threads=THREADS)
    _check_y(m.gemv(xf.cuda()).cpu().numpy(), yref32)
    dec = m.decode()
    want = (codes_d.float() * torch.from_numpy(step).cuda()).bfloat16()
    assert torch.equal(dec, want)


QWEN15B = [("q", 1536, 1536), ("k", 256, 1536), ("v", 256, 1536), ("o", 1536, 1536),
           ("gate", 8960, 1536), ("up", 8960, 1536), ("down", 1536, 8960)]
PHASE = {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3}


def test_whole_qwen15b_step_plans_against_oracle(torch, rb):
    encs = []
    for pi, (name, rows, cols) in enumerate(QWEN15B):
        codes = _codes(torch, rows, cols, "gauss", 4.25, seed=500 + pi).cpu().numpy()
        encs.append(rb.encode(codes, 8, 512 if cols % 512 == 0 else 640, nthreads=THREADS))
    mats, xs, steps, phases, kinds = [], [], [], [], []
    g = torch.Generator().manual_seed(8)
    for li in range(28):
        for pi, (name, rows, cols) in enumerate(QWEN15B):
            step = _step(cols, "gauss", 1000 * li + pi)
            mats.append(rb.RansMatrix(encs[pi], torch.from_numpy(step)))
            xs.append(torch.randn(cols, generator=g).bfloat16().cuda())
            steps.append(step)
            phases.append(4 * li + PHASE[name])
            kinds.append(pi)
    ys_step = [torch.full((m.rows,), float("nan"), device="cuda") for m in mats]
    st = rb.RansStep(mats, xs, ys_step)
    ys_chain = [torch.full((m.rows,), float("nan"), device="cuda") for m in mats]
    ch = rb.RansChain(mats, xs, ys_chain, phases)
    for _ in range(2):
        st()
        ch()
    ch.check()
    torch.cuda.synchronize()
    for i in range(len(mats)):
        xs64 = xs[i].float().cpu().numpy().astype(np.float64) * steps[i].astype(np.float64)
        yref = orc.c_decode_gemv(encs[kinds[i]], xs64, threads=THREADS)
        _check_y(ys_step[i].cpu().numpy(), yref)
        _check_y(ys_chain[i].cpu().numpy(), yref)
