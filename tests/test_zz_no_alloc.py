"""rans_gemv_step_noalloc: the decoder-step launcher for callers that cannot
allocate device memory when they run a step (a framework's caching allocator
owning the pool, an allocation-free inference loop).  Its plan lives in a
fixed 256 KB device array inside librans_b200.so instead of a caller workspace.

Checked through the C ABI against the workspace entry point
(rans_gemv_step_plan + rans_gemv_step_launch) on two calls in a row, and the
oversize-plan rejection (decided from the shapes, before any GPU work).
This file is collected last on purpose.
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import golden_cases, load_case
from oracle import rans_oracle as orc

REL_L2 = 1e-3   # the GEMV tolerance used by the other parity tests


def _lib():
    import rans_b200 as rb
    lib = rb.load()
    f = lib.rans_gemv_step_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return rb, lib


def test_noalloc_rejects_oversize_plan():
    rb, lib = _lib()
    # 2^20 rows at R=1 -> 2^20 row blocks, one item each -> 131,072 eight-item
    # chunks -> a plan of about 2 MB: over the 256 KB array.
    d = rb.RansGemvDesc(None, None, None, None, None, None, -1, 1 << 20, 64, 64, 0)
    arr = (rb.RansGemvDesc * 1)(d)
    assert lib.rans_gemv_step_noalloc(ctypes.addressof(arr), 1, 1, None) == -3
    assert lib.rans_gemv_step_noalloc(ctypes.addressof(arr), 1, 3, None) == -1
    assert lib.rans_gemv_step_noalloc(ctypes.addressof(arr), 0, 1, None) == -2


@pytest.mark.gpu
def test_noalloc_step_matches_workspace_step(cuda_ok):
    import torch
    rb, lib = _lib()
    mats, xs, refs = [], [], []
    for path in golden_cases():
        codes, enc, step, x, y, _ = load_case(path)
        if enc["R"] != 8:
            continue
        mats.append(rb.RansMatrix(enc, torch.from_numpy(step)))
        xb = torch.from_numpy(x).bfloat16()
        xs.append(xb.cuda())
        refs.append(orc.gemv(codes, step.astype(np.float64), xb.float().numpy().astype(np.float64)))
    codes = orc.synth_codes(1024, 1536, 4.25, "gauss", seed=3)
    step = (0.01 * np.random.default_rng(3).uniform(0.5, 1.5, 1536)).astype(np.float32)
    mats.append(rb.RansMatrix(rb.encode(codes, 8, 512), torch.from_numpy(step)))
    xb = torch.randn(1536, generator=torch.Generator().manual_seed(3)).bfloat16()
    xs.append(xb.cuda())
    refs.append(orc.gemv(codes, step.astype(np.float64), xb.float().numpy().astype(np.float64)))

    # existing entry point (caller-allocated workspace)
    ys_ws = [torch.full((m.rows,), float("nan"), device="cuda") for m in mats]
    rb.RansStep(mats, xs, ys_ws)()
    torch.cuda.synchronize()
    want = [y.cpu().numpy() for y in ys_ws]

    ys = [torch.empty(m.rows, device="cuda") for m in mats]
    arr = (rb.RansGemvDesc * len(mats))(*[m.desc(x, y) for m, x, y in zip(mats, xs, ys)])
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        for y in ys:
            y.fill_(float("nan"))
        rc = lib.rans_gemv_step_noalloc(ctypes.addressof(arr), len(mats), 8, stream)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        for y, w, r in zip(ys, want, refs):
            got = y.cpu().numpy()
            assert orc.rel_l2(got, w) <= REL_L2
            assert orc.rel_l2(got, r) <= REL_L2
