"""The reference's own kernel benchmark on B200: the 18 (shape, bits, R, C)
records of its results/kernel_bench.json (kernel/bench.py:82-126 picked R
and C per shape on its own GPU), run here against the reference's kernel
compiled unmodified for sm_100a (oracle/_ref/librans_ref.so) through the same
C entry point and device buffers, with bf16 cuBLAS beside them.

Codes: kernel/bench.py:26-35 (Laplace, entropy bisection; restated in the
oracle); steps rand*0.01+0.005 (bench.py:92); fp32 x.  With RANS_PERF_OUT set
every record is appended there as a JSON line."""
import ctypes
import json
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import rans_oracle as orc

pytestmark = pytest.mark.gpu

# (name, rows, cols, bits, R, C) as in the reference's kernel_bench records
RECORDS = [
    ("1.5B qkv", 2048, 1536, 2.0, 4, 512), ("1.5B qkv", 2048, 1536, 3.0, 4, 512),
    ("1.5B qkv", 2048, 1536, 4.0, 4, 512),
    ("1.5B gate_up", 17920, 1536, 2.0, 4, 1536), ("1.5B gate_up", 17920, 1536, 3.0, 8, 1536),
    ("1.5B gate_up", 17920, 1536, 4.0, 8, 1536),
    ("1.5B down", 1536, 8960, 2.0, 8, 8960), ("1.5B down", 1536, 8960, 3.0, 8, 8960),
    ("1.5B down", 1536, 8960, 4.0, 8, 8960),
    ("27B attn", 5120, 5120, 2.0, 16, 1024), ("27B attn", 5120, 5120, 3.0, 16, 512),
    ("27B attn", 5120, 5120, 4.0, 16, 512),
    ("27B gate_up", 34816, 5120, 2.0, 4, 512), ("27B gate_up", 34816, 5120, 3.0, 4, 512),
    ("27B gate_up", 34816, 5120, 4.0, 4, 512),
    ("27B down", 5120, 17408, 2.0, 4, 512), ("27B down", 5120, 17408, 3.0, 4, 512),
    ("27B down", 5120, 17408, 4.0, 4, 512),
]


def _ref_lib():
    path = os.path.join(ROOT, "oracle", "_ref", "librans_ref.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/librans_ref.so not built")
    lib = ctypes.CDLL(path)
    lib.launch_rans_gemv.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    lib.launch_rans_gemv.restype = ctypes.c_int
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


@pytest.mark.parametrize("name,rows,cols,bits,R,C", RECORDS, ids=[f"{r[0]}-{r[3]}b".replace(" ", "_") for r in RECORDS])
def test_reference_kernel_bench_record(cuda_ok, name, rows, cols, bits, R, C):
    import torch
    import rans_b200 as rb
    mine, ref = rb.load(), _ref_lib()
    codes = orc.synth_codes(rows, cols, bits, "laplace", seed=rows)
    enc = rb.encode(codes, R, C)
    g = torch.Generator().manual_seed(rows)
    step = torch.rand(cols, generator=g) * 0.01 + 0.005
    nbytes = enc["words"].nbytes + enc["offs"].nbytes
    ncop = max(1, min(16, int(400e6 // nbytes)))
    mats = [rb.RansMatrix(enc, step) for _ in range(ncop)]
    x = torch.randn(cols, generator=g).cuda()
    xs = (x * mats[0].step).contiguous()
    y = torch.zeros(rows, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def gemv(lib, m):
        return lambda: lib.launch_rans_gemv(R, m.words.data_ptr(), m.offs.data_ptr(), m.table.data_ptr(),
                                            xs.data_ptr(), y.data_ptr(), rows, cols, C, st)

    y.zero_(); gemv(mine, mats[0])(); torch.cuda.synchronize(); ya = y.clone()
    y.zero_(); gemv(ref, mats[0])(); torch.cuda.synchronize(); yb = y.clone()
    assert orc.rel_l2(ya.cpu().numpy(), yb.cpu().numpy()) < 1e-5
    it = 30 if rows * cols < 5e7 else 10
    t_mine = _time_us(torch, [gemv(mine, m) for m in mats], it)
    t_ref = _time_us(torch, [gemv(ref, m) for m in mats], it)
    xb = x.bfloat16()
    W = (torch.from_numpy(codes).float() * step).bfloat16().cuda()
    t_cublas = _time_us(torch, [lambda: torch.nn.functional.linear(xb, W)], it)
    bits_total = 8.0 * (nbytes + enc["table"].nbytes) / (rows * cols)
    rec = dict(name=name, shape=f"{rows}x{cols}", bits=bits, R=R, C=C, bits_total=round(bits_total, 3),
               gemv_us=round(t_mine, 2), ref_gemv_us=round(t_ref, 2), speedup=round(t_ref / t_mine, 2),
               cublas_bf16_us=round(t_cublas, 2), vs_cublas=round(t_cublas / t_mine, 3),
               eff_bf16_gbs=round(2 * rows * cols / t_mine / 1e3, 1))
    out = os.environ.get("RANS_PERF_OUT")
    if out:
        with open(out, "a") as f:
            f.write(json.dumps(rec) + "\n")
    assert t_mine < t_ref, rec
