"""Speed against the reference's own CUDA kernels on the same B200.

The reference library (kernel/rans_gemv.cu compiled unmodified for sm_100a
into oracle/_ref/librans_ref.so by oracle/Makefile) and librans_b200.so are
driven through the SAME three C entry points with the SAME device buffers;
kernel time is taken with CUDA events over a rotation of matrix copies larger
than L2.  Results are checked for equality first.  With RANS_PERF_OUT set the
timings are written there as JSON lines.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import rans_oracle as orc

pytestmark = pytest.mark.gpu

SHAPES = [  # rows, cols, R, C, dist, bits
    (1536, 1536, 8, 512, "laplace", 3.25),
    (8960, 1536, 8, 512, "gauss", 4.25),      # config 2 gate/up
    (1536, 8960, 8, 640, "gauss", 4.25),      # config 2 down
    (28672, 8192, 8, 512, "laplace", 2.25),   # config 5 gate/up
    (8192, 28672, 8, 512, "laplace", 2.25),   # config 5 down
    (1536, 1536, 8, 1536, "laplace", 3.25),   # one column block (C = cols), as the reference's sweep picks
]


def _ref_lib():
    path = os.path.join(ROOT, "oracle", "_ref", "librans_ref.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/librans_ref.so not built")
    lib = ctypes.CDLL(path)
    for f in (lib.launch_rans_gemv, lib.launch_rans_decode):
        f.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
        f.restype = ctypes.c_int
    lib.launch_int4_gemv.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 2 + [ctypes.c_void_p]
    lib.launch_int4_gemv.restype = ctypes.c_int
    return lib


def _time_us(torch, fns, iters):
    for f in fns[:3]:
        f()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(iters):
        fns[i % len(fns)]()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3


@pytest.mark.parametrize("rows,cols,R,C,dist,bits", SHAPES)
def test_faster_than_reference_kernels(cuda_ok, rows, cols, R, C, dist, bits):
    import torch
    import rans_b200 as rb
    mine, ref = rb.load(), _ref_lib()
    base = orc.synth_codes(min(rows, 4096), cols, bits, dist, seed=rows + cols)
    codes = np.tile(base, (-(-rows // base.shape[0]), 1))[:rows]
    enc = rb.encode(codes, R, C)
    g = torch.Generator().manual_seed(rows)
    step = torch.rand(cols, generator=g) * 0.01 + 0.005
    ncop = max(1, min(32, int(400e6 // (enc["words"].nbytes + enc["offs"].nbytes))))
    mats = [rb.RansMatrix(enc, step) for _ in range(ncop)]
    x = torch.randn(cols, generator=g).cuda()
    xs = (x * mats[0].step).contiguous()
    y = torch.zeros(rows, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def gemv(lib, m):
        return lambda: lib.launch_rans_gemv(R, m.words.data_ptr(), m.offs.data_ptr(), m.table.data_ptr(),
                                            xs.data_ptr(), y.data_ptr(), rows, cols, C, st)

    # equality first: same inputs, both libraries (y zeroed: reference contract)
    y.zero_(); gemv(mine, mats[0])(); torch.cuda.synchronize(); ya = y.clone()
    y.zero_(); gemv(ref, mats[0])(); torch.cuda.synchronize(); yb = y.clone()
    assert orc.rel_l2(ya.cpu().numpy(), yb.cpu().numpy()) < 1e-5
    # the fused bf16 entry point (step applied in-kernel) on the same weights
    xb = x.bfloat16()
    xsb = (xb.float() * mats[0].step).contiguous()
    y.zero_()
    ref.launch_rans_gemv(R, mats[0].words.data_ptr(), mats[0].offs.data_ptr(), mats[0].table.data_ptr(),
                         xsb.data_ptr(), y.data_ptr(), rows, cols, C, st)
    yc = mats[0].gemv_bf16(xb, torch.full((rows,), float("nan"), device="cuda"))
    torch.cuda.synchronize()
    assert orc.rel_l2(yc.cpu().numpy(), y.cpu().numpy()) < 1e-5
    out_a = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
    out_b = torch.empty_like(out_a)

    def decode(lib, m, out):
        return lambda: lib.launch_rans_decode(R, m.words.data_ptr(), m.offs.data_ptr(), m.table.data_ptr(),
                                              m.step.data_ptr(), out.data_ptr(), rows, cols, C, st)
    decode(mine, mats[0], out_a)(); decode(ref, mats[0], out_b)(); torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)

    it = 40 if rows * cols < 1e8 else 12
    t_mine = _time_us(torch, [gemv(mine, m) for m in mats], it)
    t_ref = _time_us(torch, [gemv(ref, m) for m in mats], it)
    t_bf16 = _time_us(torch, [(lambda m=m: mine.rans_gemv_bf16(R, m.words.data_ptr(), m.offs.data_ptr(),
                                                            m.table.data_ptr(), xb.data_ptr(), m.step.data_ptr(),
                                                            y.data_ptr(), rows, cols, C, m.nwords, st))
                               for m in mats], it)
    t_dec = _time_us(torch, [decode(mine, m, out_a) for m in mats], max(4, it // 4))
    t_dec_ref = _time_us(torch, [decode(ref, m, out_b) for m in mats], max(4, it // 4))
    q = np.clip(codes, -8, 7)
    m4 = rb.Int4Matrix(q, step)
    y4 = torch.empty(rows, device="cuda")
    x4 = (x * m4.step).contiguous()
    t_i4 = _time_us(torch, [lambda: mine.launch_int4_gemv(m4.w.data_ptr(), x4.data_ptr(), y4.data_ptr(), rows,
                                                          cols, st)], it)
    t_i4_ref = _time_us(torch, [lambda: ref.launch_int4_gemv(m4.w.data_ptr(), x4.data_ptr(), y4.data_ptr(), rows,
                                                             cols, st)], it)
    W = (torch.from_numpy(codes).float() * step).bfloat16().cuda()
    t_cublas = _time_us(torch, [lambda: torch.nn.functional.linear(xb, W)], it)
    rec = dict(shape=f"{rows}x{cols}", R=R, C=C, dist=dist, bits=bits,
               gemv_us=round(t_mine, 2), ref_gemv_us=round(t_ref, 2), gemv_speedup=round(t_ref / t_mine, 2),
               gemv_bf16_us=round(t_bf16, 2),
               decode_us=round(t_dec, 2), ref_decode_us=round(t_dec_ref, 2),
               int4_us=round(t_i4, 2), ref_int4_us=round(t_i4_ref, 2), cublas_bf16_us=round(t_cublas, 2),
               tsym_per_s=round(rows * cols / t_mine / 1e6, 3))
    out = os.environ.get("RANS_PERF_OUT")
    if out:
        with open(out, "a") as f:
            f.write(json.dumps(rec) + "\n")
    assert t_mine < t_ref, rec
    assert t_i4 < t_i4_ref, rec
    assert t_dec < 1.1 * t_dec_ref, rec
