"""Host-side product code on CPU: the C++ encoder against the reference's own
outputs, and the C-ABI library's exported symbols against include/*.h."""
import ctypes
import glob
import json
import os
import re
import hashlib

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from conftest import GOLDEN, ROOT, golden_cases, load_case
import rans_b200 as rb
from oracle import rans_oracle as orc

CASES = golden_cases()
IDS = [os.path.basename(p)[:-4] for p in CASES]


@pytest.fixture(scope="module")
def lib():
    return rb.build()


def header_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:int|int64_t|size_t|void)\s+\**\s*(\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_reference_entry_points():
    syms = header_symbols()
    for name in ("launch_rans_gemv", "launch_rans_decode", "launch_int4_gemv"):
        assert name in syms


def test_library_exports_every_header_symbol(lib):
    handle = ctypes.CDLL(rb.LIB)
    missing = [s for s in header_symbols() if not hasattr(handle, s)]
    assert not missing, f"not exported: {missing}"
    assert lib.rans_b200_abi_version() == rb.ABI_VERSION


def test_reference_argtypes_bind(lib):
    # the reference's build() binds exactly these; they must be present and callable types
    for f in (lib.launch_rans_gemv, lib.launch_rans_decode):
        assert len(f.argtypes) == 10
    assert len(lib.launch_int4_gemv.argtypes) == 6


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_cpp_encoder_bit_exact(lib, path):
    codes, enc, *_, bits = load_case(path)
    for nt in (1, 3):
        mine = rb.encode(codes, enc["R"], enc["C"], nthreads=nt)
        assert np.array_equal(mine["table"], enc["table"])
        assert np.array_equal(mine["offs"], enc["offs"])
        assert np.array_equal(mine["words"], enc["words"])
    np.testing.assert_allclose([mine["bits_payload"], mine["bits_state_offs"], mine["bits_table"],
                                mine["entropy_model"]], bits, rtol=1e-12, atol=1e-9)


def test_cpp_encoder_config1(lib):
    meta = json.load(open(os.path.join(GOLDEN, "config1.json")))
    codes = orc.synth_codes(meta["rows"], meta["cols"], meta["target_bits"], meta["dist"], meta["seed"])
    enc = rb.encode(codes, meta["R"], meta["C"])
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert sha(enc["words"]) == meta["sha_words"]
    assert sha(enc["offs"]) == meta["sha_offs"]
    assert sha(enc["table"]) == meta["sha_table"]


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_cpp_table(lib, path):
    codes, enc, *_ = load_case(path)
    f, c, t = rb.build_table(orc.codes_to_symbols(codes))
    f2, c2, t2 = orc.build_table(orc.codes_to_symbols(codes))
    assert np.array_equal(t, enc["table"]) and np.array_equal(f, f2) and np.array_equal(c, c2)


def test_encoder_random_shapes_against_oracle(lib):
    rng = np.random.default_rng(5)
    for trial in range(6):
        R = int(rng.choice([1, 2, 4, 8, 16]))
        C = int(32 * rng.integers(1, 6))
        rows, cols = R * int(rng.integers(1, 5)), C * int(rng.integers(1, 4))
        codes = np.clip(np.round(rng.laplace(0, rng.uniform(0.3, 8), (rows, cols))), -128, 127).astype(np.int32)
        codes.flat[0] = 1  # never single-symbol
        codes.flat[-1] = -1
        a = rb.encode(codes, R, C, nthreads=2)
        b = orc.encode(codes, R, C)
        for k in ("words", "offs", "table"):
            assert np.array_equal(a[k], b[k]), (trial, k)


@settings(max_examples=40, deadline=None)
@given(data=st.data())
def test_encoder_edge_distributions_against_oracle(lib, data):
    """The C++ producer byte-for-byte against the oracle restatement of the
    reference encoder on the distributions that stress the 12-bit frequency
    normalisation: two symbols only, the alphabet's two extremes only, one
    dominant symbol with many singletons (each must keep frequency >= 1), the
    whole alphabet uniformly, and Laplacian codes of any scale."""
    R = data.draw(st.sampled_from([1, 2, 4, 8, 16]))
    C = 32 * data.draw(st.integers(1, 4))
    rows, cols = R * data.draw(st.integers(1, 4)), C * data.draw(st.integers(1, 3))
    kind = data.draw(st.sampled_from(["two", "extremes", "dominant", "uniform", "laplace"]))
    rng = np.random.default_rng(data.draw(st.integers(0, 2**31 - 1)))
    if kind == "two":
        a, b = sorted(rng.choice(256, 2, replace=False) - 128)
        codes = np.where(rng.random((rows, cols)) < rng.uniform(0.001, 0.999), a, b)
    elif kind == "extremes":
        codes = np.where(rng.random((rows, cols)) < 0.5, -128, 127)
    elif kind == "dominant":
        codes = np.zeros((rows, cols), np.int64)
        k = min(rows * cols - 1, 200)
        idx = rng.choice(rows * cols, k, replace=False)
        codes.flat[idx] = rng.choice(np.r_[-128:0, 1:128], k)   # up to 200 rare symbols
    elif kind == "uniform":
        codes = rng.integers(-128, 128, (rows, cols))
    else:
        codes = np.clip(np.round(rng.laplace(0, rng.uniform(0.05, 40), (rows, cols))), -128, 127)
    codes = codes.astype(np.int32)
    if len(np.unique(codes)) < 2:                              # a single symbol cannot be coded
        codes.flat[0] = codes.flat[0] + (1 if codes.flat[0] < 127 else -1)
    a = rb.encode(codes, R, C, nthreads=3)
    b = orc.encode(codes, R, C)
    for k in ("words", "offs", "table"):
        assert np.array_equal(a[k], b[k]), (kind, k)


def test_encoder_errors(lib):
    with pytest.raises(AssertionError):
        rb.encode(np.zeros((8, 64), np.int32), 8, 64)          # single symbol
    with pytest.raises(ValueError):
        rb.encode(np.full((8, 64), 300), 8, 64)                # out of alphabet
    with pytest.raises(AssertionError):
        rb.encode(np.ones((8, 64)), 3, 64)                     # rows % R
    assert lib.rans_encode_bound(8, 60, 8, 60) == -2


def test_launchers_reject_bad_arguments_without_launching(lib):
    # argument checks happen before any CUDA call, so these run without a GPU
    assert lib.launch_rans_gemv(3, None, None, None, None, None, 6, 64, 64, None) == -1
    assert lib.launch_rans_gemv(8, None, None, None, None, None, 12, 64, 64, None) == -2
    assert lib.launch_rans_decode(8, None, None, None, None, None, 16, 64, 48, None) == -2
    assert lib.launch_int4_gemv(None, None, None, 4, 40, None) == -2
    assert lib.rans_gemv_bf16(5, None, None, None, None, None, None, 8, 64, 64, -1, None) == -1


def test_planning_reaches_cuda_for_every_mode():
    """Host-side planning of every launch mode (row mode, column mode, split
    small and large matrices, every R) runs to its first CUDA call without
    crashing.  Run in a child process with no device visible, so that call
    fails with a CUDA error code and nothing is launched (the pointers are
    never dereferenced; the bf16 entry only checks that `step` is non-null)."""
    import subprocess
    import sys
    from conftest import PKG
    code = f"""
import sys
sys.path.insert(0, {PKG!r})
import rans_b200 as rb
lib = rb.load()
shapes = [(8, 64, 64), (8, 1024, 64), (64, 1024, 1024), (1536, 1536, 512), (1536, 8960, 640),
          (28672, 8192, 512), (8192, 28672, 512)]
for rows, cols, C in shapes:
    for R in (1, 2, 4, 8, 16):
        if rows % R:
            continue
        rc = (lib.launch_rans_gemv(R, None, None, None, None, None, rows, cols, C, None),
              lib.rans_gemv_bf16(R, None, None, None, None, 256, None, rows, cols, C, -1, None),
              lib.launch_rans_decode(R, None, None, None, None, None, rows, cols, C, None))
        assert all(v > 0 for v in rc), (rows, cols, C, R, rc)
print("planned ok")
"""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "planned ok" in r.stdout, (r.returncode, r.stdout[-1000:], r.stderr[-2000:])


def _descs(n, rows, cols, C, bf16_x, nwords=1 << 20):
    arr = (rb.RansGemvDesc * n)()
    for i in range(n):
        # pointers are never dereferenced by the workspace query
        arr[i] = rb.RansGemvDesc(256, 256, 256, 256, 256 if bf16_x else None, 256, nwords, rows, cols, C, 0)
    return arr


def test_step_workspace_layout_without_gpu(lib):
    """Host-side step planning: a multi-wave launch with bf16 activations gets
    a prescaled fp32 copy of every activation vector in its workspace; a
    short (split) launch and fp32 activations do not."""
    big_bf16 = lib.rans_gemv_step_workspace_bytes(_descs(6, 8960, 1536, 512, True), 6, 8)
    big_f32 = lib.rans_gemv_step_workspace_bytes(_descs(6, 8960, 1536, 512, False), 6, 8)
    assert big_bf16 > 0 and big_f32 > 0
    assert big_bf16 - big_f32 >= 6 * 1536 * 4          # x' copies + their job table
    small_bf16 = lib.rans_gemv_step_workspace_bytes(_descs(1, 256, 1536, 512, True), 1, 8)
    small_f32 = lib.rans_gemv_step_workspace_bytes(_descs(1, 256, 1536, 512, False), 1, 8)
    assert small_bf16 == small_f32
    assert lib.rans_gemv_step_workspace_bytes(_descs(1, 12, 1536, 512, True), 1, 8) == -2   # rows % R
    assert lib.rans_gemv_step_workspace_bytes(_descs(1, 256, 1536, 512, True), 1, 3) == -1  # bad R


def _chain_describe(lib, shapes, phases, R, steps, nbits=None):
    """Chunk records of the chain planner for `shapes` [(rows, cols, C)]."""
    import ctypes
    n = len(shapes)
    arr = (rb.RansGemvDesc * n)()
    for i, (rows, cols, C) in enumerate(shapes):
        bits = 2.6 if nbits is None else nbits[i]               # default ~2.25 b/w payload + overhead
        nwords = int(rows * cols * bits / 16) + 8
        arr[i] = rb.RansGemvDesc(256, 256, 256, 256, 256 if steps[i] else None, 256, nwords, rows, cols, C, 0)
    ph = (ctypes.c_int * n)(*phases)
    nc = lib.rans_gemv_chain_describe(ctypes.addressof(arr), ctypes.addressof(ph), n, R, None, 0)
    assert nc > 0, nc
    out = (ctypes.c_int32 * (8 * nc))()
    assert lib.rans_gemv_chain_describe(ctypes.addressof(arr), ctypes.addressof(ph), n, R, out, nc) == nc
    return np.frombuffer(out, dtype=np.int32).reshape(nc, 8).copy()


@pytest.mark.parametrize("case", ["llama70b", "llama70b_rank_of_2", "llama70b_rank_of_8", "qwen_R16", "qwen_R1_fp32"])
def test_chain_plan_covers_every_tile_once_without_gpu(lib, case):
    """The chain planner's work list (rans_gemv_chain_describe, no GPU): every
    tile of every matrix is decoded by exactly one item, whatever mix of whole
    items, latency splits and half-size tail items the planner chose; phases
    are handed out in order, each matrix in its own phase (plus one when an
    activation prescale phase runs in front); a chunk holds at most one item
    per warp; and every bf16-activation matrix gets its columns prescaled
    exactly once, one phase before its own."""
    h, kv, f = 8192, 1024, 28672
    llama = [(h, h, 512), (kv, h, 512), (kv, h, 512), (h, h, 512), (f, h, 512), (f, h, 512), (h, f, 512)]
    qwen = [(1536, 1536, 512), (256, 1536, 512), (256, 1536, 512), (1536, 1536, 512),
            (8960, 1536, 512), (8960, 1536, 512), (1536, 8960, 640)]
    phase_of = [0, 0, 0, 1, 2, 2, 3]
    layer, R, world, layers, bf16 = {
        "llama70b": (llama, 8, 1, 2, True), "llama70b_rank_of_2": (llama, 8, 2, 2, True),
        "llama70b_rank_of_8": (llama, 8, 8, 2, True), "qwen_R16": (qwen, 16, 1, 3, True),
        "qwen_R1_fp32": (qwen, 1, 1, 2, False)}[case]
    shapes = [(rows // world, cols, C) for _ in range(layers) for rows, cols, C in layer]
    phases = [4 * l + p for l in range(layers) for p in phase_of]
    steps = [bf16 and (i % 2 == 0 or p > 0) for i, p in enumerate(phases)]   # mixed bf16 / fp32 x
    _check_chain_plan(_chain_describe(lib, shapes, phases, R, steps), shapes, phases, R, steps)


def _check_chain_plan(rec, shapes, phases, R, steps):
    kphase, mat, kind, first, count, tiles, streams, nseg = rec.T
    assert (np.diff(kphase) >= 0).all()                                   # phases in order
    shift = 1 if any(s for s, p in zip(steps, phases) if p == 0) else 0
    dec = kind == 0
    assert (kphase[dec] == np.array(phases)[mat[dec]] + shift).all()
    assert ((count[dec] >= 1) & (count[dec] <= 8)).all()
    assert ((streams[dec] >= 1) & (streams[dec] <= 4) & (streams[dec] <= tiles[dec])).all()
    for i, (rows, cols, C) in enumerate(shapes):
        nrb, ncb = rows // R, cols // C
        cov = np.zeros((nrb, ncb), dtype=np.int32)
        for c in np.nonzero(dec & (mat == i))[0]:
            for it in range(first[c], first[c] + count[c]):
                rbk, seg = divmod(it, nseg[c])
                cov[rbk, seg * tiles[c]:min(ncb, (seg + 1) * tiles[c])] += 1
        assert (cov == 1).all(), f"matrix {i}: tiles decoded {cov.min()}..{cov.max()} times"
        pre = np.nonzero((kind == 1) & (mat == i))[0]
        if not steps[i]:
            assert len(pre) == 0
            continue
        colcov = np.zeros(cols, dtype=np.int32)
        for c in pre:
            assert kphase[c] == phases[i] + shift - 1
            colcov[first[c]:first[c] + count[c]] += 1
        assert (colcov == 1).all()


@settings(max_examples=60, deadline=None)
@given(data=st.data())
def test_chain_plan_random_shapes_without_gpu(lib, data):
    """The same invariants on random chains: tile heights R 1-16, tile widths C
    32-768, one to twenty column tiles, matrices of one row block up to
    hundreds, 0.5-8 bits per weight (the stage holds fewer or more tiles per
    pass), phases of any size, bf16 and fp32 activations mixed."""
    R = data.draw(st.sampled_from([1, 2, 4, 8, 16]))
    n = data.draw(st.integers(1, 9))
    shapes, nbits = [], []
    for _ in range(n):
        C = 32 * data.draw(st.integers(1, 24))
        shapes.append((R * data.draw(st.integers(1, 300)), C * data.draw(st.integers(1, 20)), C))
        nbits.append(data.draw(st.floats(0.5, 8.0)))
    raw = [data.draw(st.integers(0, n - 1)) for _ in range(n)]
    used = sorted(set(raw))
    phases = [used.index(v) for v in raw]                 # numbered 0..P-1 without gaps
    steps = [data.draw(st.booleans()) for _ in range(n)]
    rec = _chain_describe(lib, shapes, phases, R, steps, nbits)
    _check_chain_plan(rec, shapes, phases, R, steps)


def test_chain_workspace_layout_without_gpu(lib):
    """Host-side chain planning: phases must be numbered 0..P-1 without gaps;
    the workspace holds the descriptors, the chunks of every phase, the phase
    table and the control block, and never the prescaled activations (a
    phase may read what the previous one wrote)."""
    import ctypes
    layer = [(1536, 1536, 512), (256, 1536, 512), (256, 1536, 512), (1536, 1536, 512),
             (8960, 1536, 512), (8960, 1536, 512), (1536, 8960, 640)]
    phase_of = [0, 0, 0, 1, 2, 2, 3]
    for layers in (1, 4):
        n = 7 * layers
        arr = (rb.RansGemvDesc * n)()
        for i in range(n):
            rows, cols, C = layer[i % 7]
            arr[i] = rb.RansGemvDesc(256, 256, 256, 256, 256, 256, 1 << 20, rows, cols, C, 0)
        ph = (ctypes.c_int * n)(*[4 * (i // 7) + phase_of[i % 7] for i in range(n)])
        b = lib.rans_gemv_chain_workspace_bytes(ctypes.addressof(arr), ctypes.addressof(ph), n, 8)
        assert b > 0
        if layers == 1:
            one = b
    assert b > 3 * one                                   # grows with the layers
    bad = (ctypes.c_int * 7)(0, 0, 0, 2, 2, 2, 3)         # phase 1 missing
    assert lib.rans_gemv_chain_workspace_bytes(ctypes.addressof(arr), ctypes.addressof(bad), 7, 8) == -2
    neg = (ctypes.c_int * 7)(0, 0, 0, -1, 1, 1, 2)
    assert lib.rans_gemv_chain_workspace_bytes(ctypes.addressof(arr), ctypes.addressof(neg), 7, 8) == -2
    ok = (ctypes.c_int * 7)(*phase_of)
    assert lib.rans_gemv_chain_workspace_bytes(ctypes.addressof(arr), ctypes.addressof(ok), 7, 3) == -1
    # a bad timeout or rank description is refused before any CUDA call
    assert lib.rans_gemv_chain_plan(ctypes.addressof(arr), ctypes.addressof(ok), 7, 8, None, 0, None, 0,
                                    None, None) == -2
    sync = rb.RansChainSync(9, 0, 256, 256, 256)
    assert lib.rans_gemv_chain_plan(ctypes.addressof(arr), ctypes.addressof(ok), 7, 8, ctypes.addressof(sync),
                                    1000, None, 0, None, None) == -2
