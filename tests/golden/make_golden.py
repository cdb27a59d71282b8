"""Generate the golden fixtures in this folder from the REFERENCE implementation.

Run once where the reference checkout is available, naming it (required):

    python tests/golden/make_golden.py <path to the reference checkout>

It imports the reference's own kernel/rans.py (encoder, table, reference
decoder) and kernel/bench.py (synthetic code generator) unchanged and records
their outputs.  The GPU box never runs this script; tests read the .npz /
.json files it wrote.

Fixtures:
  * bench_test_*.npz  -- the four configurations of kernel/bench.py:41-42
    (seed = rows, Laplace), with the step vector drawn exactly as
    kernel/bench.py:40,47 does (torch.manual_seed(0); torch.rand(cols) + 0.5)
    and a seeded numpy x; y is the float64 dequantise-then-matvec.
  * edge_*.npz        -- edge cases: Gaussian 4.25 b, extreme symbols -128/127,
    all 256 symbols present, a dominant symbol (table fix-up from above),
    R=16 with C=cols, R=1 C=32, and the int4-range codes of kernel/bench.py:60.
  * config1.json      -- BASELINE config 1 (1536x1536 Laplace H~3.25, R=8,
    C=512): SHA-256 digests of codes/words/offs/table plus the reference y.
"""
import hashlib
import json
import os
import sys

import numpy as np

if len(sys.argv) != 2 or not os.path.isfile(os.path.join(sys.argv[1], "kernel", "rans.py")):
    sys.exit("usage: make_golden.py <path to the reference checkout (holding kernel/rans.py)>")
REF = os.path.abspath(sys.argv[1])
sys.path.insert(0, os.path.join(REF, "kernel"))
import rans  # noqa: E402  (the reference's kernel/rans.py)
import bench  # noqa: E402  (the reference's kernel/bench.py)
import torch  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def save_case(name, codes, R, C, step, x):
    enc = rans.encode(codes, R, C)
    dec = rans.decode_ref(enc)
    assert np.array_equal(dec, codes)
    y = (codes.astype(np.float64) * step.astype(np.float64)[None, :]) @ x.astype(np.float64)
    np.savez_compressed(
        os.path.join(OUT, f"{name}.npz"),
        codes=codes.astype(np.int16), words=enc["words"], offs=enc["offs"], table=enc["table"],
        R=R, C=C, step=step.astype(np.float32), x=x.astype(np.float32), y=y,
        bits=np.array([enc["bits_payload"], enc["bits_state_offs"], enc["bits_table"],
                       enc["entropy_model"]]))
    print(f"{name}: {codes.shape} R={R} C={C} words={enc['words'].size} "
          f"payload={enc['bits_payload']:.3f} b/w")


def main():
    # kernel/bench.py:38-56 -- same seeds, same step draws
    torch.manual_seed(0)
    for (rows, cols, R, C, bits) in [(64, 256, 4, 256, 3.0), (128, 512, 8, 128, 2.0),
                                     (256, 1024, 16, 512, 4.0), (32, 64, 1, 32, 1.0)]:
        codes = bench.synth_codes(rows, cols, bits, seed=rows)
        step = (torch.rand(cols) + 0.5).numpy()
        x = np.random.default_rng(rows + 1).standard_normal(cols).astype(np.float32)
        save_case(f"bench_test_{rows}x{cols}_R{R}_C{C}", codes, R, C, step, x)

    rng = np.random.default_rng(2024)
    # Gaussian at ~4.25 bits (BASELINE config 2 distribution), R=8 C=512
    codes = bench.synth_codes(256, 1536, 4.25, dist="gauss", seed=7)
    save_case("edge_gauss425_256x1536_R8_C512", codes, 8, 512,
              (0.01 * rng.uniform(0.5, 1.5, 1536)).astype(np.float32),
              rng.standard_normal(1536).astype(np.float32))
    # Laplace 2.25 bits with log-normal per-column steps (config 3), R=16 C=512
    codes = bench.synth_codes(256, 1024, 2.25, dist="laplace", seed=9)
    save_case("edge_lap225_256x1024_R16_C512", codes, 16, 512,
              (0.01 * np.exp(rng.normal(0, 0.5, 1024))).astype(np.float32),
              rng.standard_normal(1024).astype(np.float32))
    # extreme symbols -128 and 127 present
    codes = np.clip(np.round(rng.laplace(0, 3, (64, 512))), -20, 20).astype(np.int32)
    codes[3, 5] = -128
    codes[10, 100] = 127
    codes[63, 511] = -128
    save_case("edge_extreme_64x512_R4_C256", codes, 4, 256,
              rng.uniform(0.5, 1.5, 512).astype(np.float32),
              rng.standard_normal(512).astype(np.float32))
    # all 256 symbols present (uniform): exercises the fix-up loop
    codes = rng.integers(-128, 128, (128, 512)).astype(np.int32)
    save_case("edge_uniform256_128x512_R8_C128", codes, 8, 128,
              rng.uniform(0.5, 1.5, 512).astype(np.float32),
              rng.standard_normal(512).astype(np.float32))
    # one dominant symbol (frequency near 4095): fix-up from above
    codes = np.zeros((64, 256), np.int32)
    idx = rng.choice(codes.size, 40, replace=False)
    codes.flat[idx] = rng.choice([-3, -1, 1, 2, 5], 40)
    save_case("edge_dominant_64x256_R2_C64", codes, 2, 64,
              rng.uniform(0.5, 1.5, 256).astype(np.float32),
              rng.standard_normal(256).astype(np.float32))
    # R=16, C = cols (single column block, plain stores in the reference kernel)
    codes = bench.synth_codes(128, 768, 3.25, dist="laplace", seed=11)
    save_case("edge_R16_Ccols_128x768", codes, 16, 768,
              rng.uniform(0.5, 1.5, 768).astype(np.float32),
              rng.standard_normal(768).astype(np.float32))
    # R=1, C=32: one row, 32 columns per stream
    codes = bench.synth_codes(8, 128, 3.0, dist="laplace", seed=13)
    save_case("edge_R1_C32_8x128", codes, 1, 32,
              rng.uniform(0.5, 1.5, 128).astype(np.float32),
              rng.standard_normal(128).astype(np.float32))
    # the int4-range codes of kernel/bench.py:60, rANS-encoded
    codes = np.random.default_rng(1).integers(-8, 8, size=(256, 1024)).astype(np.int32)
    save_case("edge_int4range_256x1024_R8_C256", codes, 8, 256,
              rng.uniform(0.5, 1.5, 1024).astype(np.float32),
              rng.standard_normal(1024).astype(np.float32))

    # 1536x1536 Laplace ~3.25 bits, R=8 C=512 (digests only)
    codes = bench.synth_codes(1536, 1536, 3.25, dist="laplace", seed=1536)
    enc = rans.encode(codes, 8, 512)
    step = (0.01 * np.random.default_rng(1537).uniform(0.5, 1.5, 1536)).astype(np.float32)
    x = np.random.default_rng(1538).standard_normal(1536).astype(np.float32)
    y = (codes.astype(np.float64) * step.astype(np.float64)[None, :]) @ x.astype(np.float64)
    dec = rans.decode_ref(enc)
    assert np.array_equal(dec, codes)
    meta = dict(rows=1536, cols=1536, R=8, C=512, target_bits=3.25, dist="laplace", seed=1536,
                step_seed=1537, x_seed=1538,
                sha_codes=sha(codes.astype(np.int32)), sha_words=sha(enc["words"]),
                sha_offs=sha(enc["offs"]), sha_table=sha(enc["table"]),
                nwords=int(enc["words"].size), bits_payload=float(enc["bits_payload"]),
                entropy=float(bench.entropy(codes)), code_min=int(codes.min()),
                code_max=int(codes.max()), y=[float(v) for v in y])
    with open(os.path.join(OUT, "config1.json"), "w") as f:
        json.dump(meta, f)
    print(f"config1: words={enc['words'].size} H={meta['entropy']:.3f} "
          f"payload={enc['bits_payload']:.3f}")


if __name__ == "__main__":
    main()
