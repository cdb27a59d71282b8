"""The CPU oracle against the reference's own outputs (tests/golden, made by
importing the reference's kernel/rans.py and kernel/bench.py)."""
import json
import hashlib
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_cases, load_case
from oracle import rans_oracle as orc

CASES = golden_cases()
IDS = [os.path.basename(p)[:-4] for p in CASES]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_encode_matches_reference(path):
    codes, enc, *_ , bits = load_case(path)
    mine = orc.encode(codes, enc["R"], enc["C"])
    assert np.array_equal(mine["table"], enc["table"])
    assert np.array_equal(mine["offs"], enc["offs"])
    assert np.array_equal(mine["words"], enc["words"])
    np.testing.assert_allclose([mine["bits_payload"], mine["bits_state_offs"], mine["bits_table"],
                                mine["entropy_model"]], bits, rtol=0, atol=1e-12)


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_c_encoder_matches_reference(path):
    """The C restatement of the encoder (used for large shapes by bench.py's
    CPU legs and checks) writes the reference's bytes."""
    codes, enc, *_ , bits = load_case(path)
    mine = orc.c_encode(codes, enc["R"], enc["C"], threads=3)
    assert np.array_equal(mine["table"], enc["table"])
    assert np.array_equal(mine["offs"], enc["offs"])
    assert np.array_equal(mine["words"], enc["words"])
    np.testing.assert_allclose([mine["bits_payload"], mine["bits_state_offs"], mine["bits_table"],
                                mine["entropy_model"]], bits, rtol=0, atol=1e-12)


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_decoders_match_reference(path):
    codes, enc, step, x, y, _ = load_case(path)
    assert np.array_equal(orc.decode(enc), codes)
    assert np.array_equal(orc.c_decode_codes(enc), codes)
    s = len(enc["offs"]) // 2
    rows, cols = enc["shape"]
    R, C = enc["R"], enc["C"]
    st = orc.lane_order(codes, R, C)[s]
    assert np.array_equal(orc.decode_stream_scalar(enc, s), st)
    # fused C decode+dot equals the reference float64 y
    xs = x.astype(np.float64) * step.astype(np.float64)
    yc = orc.c_decode_gemv(enc, xs, threads=2)
    np.testing.assert_allclose(yc, y, rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose(orc.gemv(codes, step, x), y, rtol=1e-12, atol=1e-9)


@pytest.mark.parametrize("path", CASES, ids=IDS)
def test_c_table_matches_reference(path):
    codes, enc, *_ = load_case(path)
    f, c, t = orc.c_build_table(orc.codes_to_symbols(codes))
    assert np.array_equal(t, enc["table"])


def test_config1_digests():
    meta = json.load(open(os.path.join(GOLDEN, "config1.json")))
    codes = orc.synth_codes(meta["rows"], meta["cols"], meta["target_bits"], meta["dist"], meta["seed"])
    assert sha(codes.astype(np.int32)) == meta["sha_codes"]
    enc = orc.encode(codes, meta["R"], meta["C"])
    assert sha(enc["words"]) == meta["sha_words"]
    assert sha(orc.c_encode(codes, meta["R"], meta["C"], threads=4)["words"]) == meta["sha_words"]
    assert sha(enc["offs"]) == meta["sha_offs"]
    assert sha(enc["table"]) == meta["sha_table"]
    assert np.array_equal(orc.c_decode_codes(enc), codes)
    step = (0.01 * np.random.default_rng(meta["step_seed"]).uniform(0.5, 1.5, meta["cols"])).astype(np.float32)
    x = np.random.default_rng(meta["x_seed"]).standard_normal(meta["cols"]).astype(np.float32)
    np.testing.assert_allclose(orc.gemv(codes, step, x), meta["y"], rtol=1e-12, atol=1e-9)


def test_decoder_detects_corruption():
    """A flipped payload word must break the final-state check (kernel/rans.py:121)."""
    codes, enc, *_ = load_case(os.path.join(GOLDEN, "edge_gauss425_256x1536_R8_C512.npz"))
    bad = dict(enc)
    w = enc["words"].copy()
    w[int(enc["offs"][5]) + 4] ^= 0x5A5A
    bad["words"] = w
    with pytest.raises(ValueError):
        orc.c_decode(bad)
    with pytest.raises(ValueError):
        orc.decode(bad)


def test_degenerate_and_range_errors():
    with pytest.raises(ValueError):
        orc.encode(np.zeros((8, 64), np.int32), 8, 64)
    with pytest.raises(ValueError):
        orc.encode(np.full((8, 64), 200), 8, 64)
    with pytest.raises(ValueError):
        orc.lane_order(np.zeros((8, 64), np.uint8), 3, 64)
