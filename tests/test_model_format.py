"""Model integration on CPU: entropy-targeted quantisation (exp/quant.py:22-25,
122-146 restated), escape codes, the encoded-matrix container, and the escape
entry points' argument checks (no GPU needed)."""
import os

import numpy as np
import pytest

from oracle import rans_oracle as orc
import rans_b200 as rb
import rans_model as rm


def test_entropy_bits_known_answers():
    assert rm.entropy_bits([0, 0, 1, 1]) == pytest.approx(1.0)
    assert rm.entropy_bits([5, 5, 5]) == pytest.approx(0.0)
    assert rm.entropy_bits(np.arange(-300, 212)) == pytest.approx(9.0)   # 512 equiprobable codes
    assert rm.entropy_bits([]) == 0.0


@pytest.mark.parametrize("bits", [2.25, 3.25, 4.25, 6.0])
def test_ecsq_rtn_meets_target_entropy(bits):
    rng = np.random.default_rng(int(bits * 100))
    W = rng.standard_normal((256, 512)) * 0.02
    codes, step = rm.ecsq_rtn(W, bits)
    assert codes.dtype == np.int32 and step.dtype == np.float32 and step.shape == (512,)
    assert np.all(step > 0)
    assert abs(rm.entropy_bits(codes) - bits) < 0.02
    # per-column base multiplies the step (waterfilling form)
    base = rng.uniform(0.5, 2.0, 512)
    codes2, step2 = rm.ecsq_rtn(W, bits, base=base)
    assert np.allclose(step2 / step2[0], (base / base[0]).astype(np.float32), rtol=1e-5)
    assert abs(rm.entropy_bits(codes2) - bits) < 0.02


def _heavy(rows=64, cols=1024, seed=0):
    rng = np.random.default_rng(seed)
    return rng.standard_t(2.0, (rows, cols)) * 0.01


def test_escape_split_and_merge():
    codes, _ = rm.ecsq_rtn(_heavy(), 7.0)
    assert (np.abs(codes) > 127).any(), "heavy-tailed 7-bit codes should leave the 8-bit alphabet"
    c8, r, k, v, fill = rm.split_escapes(codes)
    assert c8.dtype == np.int8
    assert r.size == np.count_nonzero((codes < -128) | (codes > 127))
    inr = codes[(codes >= -128) & (codes <= 127)]
    assert fill == np.bincount(inr + 128).argmax() - 128
    assert np.array_equal(rm.merge_escapes(c8, r, k, v), codes)
    assert np.all(c8[r, k] == fill)
    # row-major order
    assert np.all(np.diff(r.astype(np.int64) * codes.shape[1] + k) > 0)
    with pytest.raises(ValueError):
        rm.split_escapes(codes, fill=200)


def test_encoded_matrix_decodes_to_original_codes():
    codes, step = rm.ecsq_rtn(_heavy(64, 1024, 1), 6.5)
    m = rm.EncodedMatrix.encode(codes, step, R=8, C=512)
    assert m.n_escapes > 0
    dec = orc.decode(m.enc)                      # oracle restatement of kernel/rans.py:101-123
    assert np.array_equal(rm.merge_escapes(dec, m.esc_rows, m.esc_cols, m.esc_codes), codes)
    # the stream is exactly the reference encoding of the filled codes
    c8, *_ = rm.split_escapes(codes)
    ref = orc.encode(c8.astype(np.int64), 8, 512)
    assert np.array_equal(m.enc["words"], ref["words"]) and np.array_equal(m.enc["offs"], ref["offs"])
    assert m.bits_per_weight() > 0


def test_container_round_trip(tmp_path):
    mats = {}
    for i, (rows, cols, bits) in enumerate([(64, 1024, 6.5), (32, 512, 3.25)]):
        codes, step = rm.ecsq_rtn(_heavy(rows, cols, 10 + i), bits)
        mats[f"layer{i}.proj"] = rm.EncodedMatrix.encode(codes, step, R=8, C=512)
    path = str(tmp_path / "m.rans")
    rm.save_matrices(path, mats, meta={"model": "synthetic"})
    for mmap in (True, False):
        got, meta = rm.load_matrices(path, mmap=mmap)
        assert meta == {"model": "synthetic"}
        assert set(got) == set(mats)
        for name, m in mats.items():
            g = got[name]
            assert g.shape == m.shape and g.fill == m.fill
            assert g.enc["R"] == 8 and g.enc["C"] == 512
            for a, b in ((g.enc["words"], m.enc["words"]), (g.enc["offs"], m.enc["offs"]),
                         (g.enc["table"], m.enc["table"]), (g.step, m.step), (g.esc_rows, m.esc_rows),
                         (g.esc_cols, m.esc_cols), (g.esc_codes, m.esc_codes)):
                assert a.dtype.kind == np.asarray(b).dtype.kind and a.itemsize == np.asarray(b).itemsize
                assert np.array_equal(a, b)
            assert g.enc["bits_payload"] == pytest.approx(m.enc["bits_payload"])
    # every array 64-byte aligned in the file
    raw = open(path, "rb").read()
    hlen = int(np.frombuffer(raw[8:16], "<u8")[0])
    import json
    hdr = json.loads(raw[16:16 + hlen])
    start = (16 + hlen + 63) // 64 * 64
    for e in hdr["matrices"].values():
        for a in e["arrays"].values():
            assert (start + a["offset"]) % 64 == 0


def test_container_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.rans"
    p.write_bytes(b"NOTRANS!" + b"\0" * 32)
    with pytest.raises(ValueError):
        rm.load_matrices(str(p))
    codes, step = rm.ecsq_rtn(_heavy(32, 512, 3), 4.0)
    good = str(tmp_path / "good.rans")
    rm.save_matrices(good, {"w": rm.EncodedMatrix.encode(codes, step, R=8, C=512)})
    trunc = tmp_path / "trunc.rans"
    trunc.write_bytes(open(good, "rb").read()[:-100])
    with pytest.raises(ValueError):
        rm.load_matrices(str(trunc))


def test_escape_entry_points_check_arguments_without_gpu():
    lib = rb.build()
    assert lib.rans_escape_gemv(None, None, None, -1, None, None, None, None) == -2
    assert lib.rans_escape_gemv(None, None, None, 0, None, None, None, None) == 0
    assert lib.rans_escape_gemv(None, None, None, 4, None, None, None, None) == -2
    assert lib.rans_escape_decode(None, None, None, 0, None, None, 16, None) == 0
    assert lib.rans_escape_decode(None, None, None, 3, None, None, 0, None) == -2
    assert lib.rans_escape_decode(None, None, None, 3, None, None, 16, None) == -2
