"""CPU oracle for the tile-interleaved rANS decode-GEMV path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this file;
it is used by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` as the checker.  It restates, in numpy (and in the companion C
file ``rans_oracle.c`` for speed), the algorithm of the reference project
snuri00/vram-compression:

  * ``build_table``   follows kernel/rans.py:34-51   (12-bit static table)
  * ``lane_order``    follows kernel/rans.py:55-59   (tile/lane interleave)
  * ``encode``        follows kernel/rans.py:62-98   (32-bit state rANS encoder)
  * ``c_encode``      the same encoder in C (rans_oracle.c, OpenMP), for large shapes
  * ``decode``        follows kernel/rans.py:101-123 (reference decoder) and the
                      device step of kernel/rans_gemv.cu:32-37
  * ``synth_codes``   follows kernel/bench.py:26-35  (synthetic ECSQ codes)
  * ``gemv``          follows kernel/bench.py:52-56  (dequantise-then-matvec)

Parity is pinned: tests/golden/ holds fixtures produced by importing the
reference's own kernel/rans.py and kernel/bench.py (script
tests/golden/make_golden.py); tests/test_oracle.py checks this module and the
C restatement against every fixture, bit for bit.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

SCALE_BITS = 12
PROB_M = 1 << SCALE_BITS          # total of the 12-bit frequencies
RANS_L = 1 << 16                  # lower bound of the normalised state
SYM_OFFSET = 128                  # symbol = code + 128
PAD_WORDS = 8                     # zero words appended after the last stream

HERE = os.path.dirname(os.path.abspath(__file__))


# ----------------------------------------------------------------- symbols
def codes_to_symbols(codes: np.ndarray) -> np.ndarray:
    """Map signed integer codes in [-128, 127] to byte symbols (kernel/rans.py:65-67)."""
    s = np.asarray(codes).astype(np.int64) + SYM_OFFSET
    if s.size and (s.min() < 0 or s.max() > 255):
        raise ValueError("code outside the 8-bit alphabet [-128, 127]")
    return s.astype(np.uint8)


# ------------------------------------------------------------------- table
def build_table(sym: np.ndarray):
    """Normalised frequencies, exclusive cumulative sums and the slot table.

    Restates kernel/rans.py:34-51:
      * frequencies of present symbols are max(1, round-half-even(count*M/total));
      * while the sum differs from M the FIRST largest bin absorbs the
        difference (when shrinking, never below 1);
      * a single-symbol distribution is rejected;
      * slot entry = sym | freq << 8 | (slot - cum) << 20.
    """
    counts = np.bincount(np.asarray(sym).ravel(), minlength=256).astype(np.float64)
    total = counts.sum()
    freq = np.zeros(256, np.int64)
    nz = counts > 0
    scaled = np.round(counts[nz] * PROB_M / total)          # numpy rounds half to even
    freq[nz] = np.maximum(scaled, 1).astype(np.int64)
    while True:
        gap = PROB_M - int(freq.sum())
        if gap == 0:
            break
        top = int(np.argmax(freq))                          # first maximum
        freq[top] += gap if gap > 0 else max(gap, 1 - int(freq[top]))
    if freq.max() >= PROB_M:
        raise ValueError("degenerate distribution (single symbol)")
    cum = np.zeros(256, np.int64)
    cum[1:] = np.cumsum(freq)[:-1]
    table = np.zeros(PROB_M, np.uint32)
    for s in np.flatnonzero(freq):
        slot = np.arange(cum[s], cum[s] + freq[s], dtype=np.int64)
        table[slot] = (s | (freq[s] << 8) | ((slot - cum[s]) << 20)).astype(np.uint32)
    return freq, cum, table


# ------------------------------------------------------------------ layout
def check_tiling(rows: int, cols: int, R: int, C: int) -> None:
    if R <= 0 or C <= 0 or rows % R or cols % C or C % 32:
        raise ValueError(f"shape {rows}x{cols} cannot be tiled by R={R}, C={C} "
                         "(need rows % R == 0, cols % C == 0, C % 32 == 0)")


def lane_order(sym: np.ndarray, R: int, C: int) -> np.ndarray:
    """(rows, cols) -> (streams, R*C/32) in stream order (kernel/rans.py:55-59).

    Stream s = (rb * ncb + cb) * 32 + lane holds, for k in 0..C/32-1 and
    r in 0..R-1, the code at row rb*R + r, column cb*C + lane + 32*k.
    """
    rows, cols = sym.shape
    check_tiling(rows, cols, R, C)
    t = sym.reshape(rows // R, R, cols // C, C // 32, 32)   # rb, r, cb, k, lane
    return t.transpose(0, 2, 4, 3, 1).reshape(-1, (C // 32) * R)


def lane_order_inverse(streams: np.ndarray, rows: int, cols: int, R: int, C: int) -> np.ndarray:
    t = streams.reshape(rows // R, cols // C, 32, C // 32, R)  # rb, cb, lane, k, r
    return t.transpose(0, 4, 1, 3, 2).reshape(rows, cols)


# ----------------------------------------------------------------- encoder
def encode(codes: np.ndarray, R: int, C: int) -> dict:
    """rANS-encode codes in the reference bitstream (kernel/rans.py:62-98).

    32-bit state starting at RANS_L, symbols pushed last-to-first; before a
    push the state emits its low 16 bits while state >= freq << 20.  Each
    stream is stored as [state >> 16, state & 0xffff] followed by the emitted
    words in reverse order; ``offs`` are word offsets of the streams, and
    PAD_WORDS zero words follow the last stream.
    """
    codes = np.asarray(codes)
    sym = codes_to_symbols(codes)
    freq, cum, table = build_table(sym)
    S = lane_order(sym, R, C)
    nstream, n = S.shape
    state = np.full(nstream, RANS_L, np.uint64)
    emitted = np.zeros((nstream, n), np.uint16)
    nemit = np.zeros(nstream, np.int64)
    fq = freq.astype(np.uint64)
    cu = cum.astype(np.uint64)
    for i in range(n - 1, -1, -1):
        f = fq[S[:, i]]
        c = cu[S[:, i]]
        hit = np.flatnonzero(state >= (f << np.uint64(20)))
        emitted[hit, nemit[hit]] = (state[hit] & np.uint64(0xFFFF)).astype(np.uint16)
        nemit[hit] += 1
        state[hit] >>= np.uint64(16)
        state = (state // f << np.uint64(SCALE_BITS)) + state % f + c
    length = nemit + 2
    offs = np.zeros(nstream, np.int64)
    offs[1:] = np.cumsum(length)[:-1]
    words = np.zeros(int(length.sum()) + PAD_WORDS, np.uint16)
    words[offs] = (state >> np.uint64(16)).astype(np.uint16)
    words[offs + 1] = (state & np.uint64(0xFFFF)).astype(np.uint16)
    # emitted words go in reverse: word j of stream s lands at offs+2+nemit-1-j
    col = np.arange(n)
    valid = col[None, :] < nemit[:, None]
    dst = offs[:, None] + 2 + nemit[:, None] - 1 - col[None, :]
    words[dst[valid]] = emitted[valid]
    nweights = codes.size
    p = freq[sym.ravel()] / PROB_M
    return dict(words=words, offs=offs.astype(np.uint32), table=table, R=R, C=C,
                shape=tuple(codes.shape),
                bits_payload=16 * (length.sum() - 2 * nstream) / nweights,
                bits_state_offs=64 * nstream / nweights,
                bits_table=32 * PROB_M / nweights,
                entropy_model=float(-np.log2(p).mean()))


# ----------------------------------------------------------------- decoder
def decode(enc: dict) -> np.ndarray:
    """Decode every stream in lock-step (numpy), return int64 codes (rows, cols).

    Per symbol (kernel/rans.py:114-120, kernel/rans_gemv.cu:32-37):
      e = table[st & 4095]; st = freq(e) * (st >> 12) + bias(e);
      if st < RANS_L: st = st << 16 | next word.
    Raises if a stream does not end in RANS_L (kernel/rans.py:121).
    """
    rows, cols = enc["shape"]
    R, C = enc["R"], enc["C"]
    check_tiling(rows, cols, R, C)
    tab = np.asarray(enc["table"]).astype(np.uint64)
    w = np.asarray(enc["words"]).astype(np.uint64)
    pos = np.asarray(enc["offs"]).astype(np.int64)
    nstream = pos.size
    n = (C // 32) * R
    st = (w[pos] << np.uint64(16)) | w[pos + 1]
    pos = pos + 2
    out = np.empty((nstream, n), np.int64)
    for i in range(n):
        e = tab[st & np.uint64(PROB_M - 1)]
        st = ((e >> np.uint64(8)) & np.uint64(0xFFF)) * (st >> np.uint64(SCALE_BITS)) + (e >> np.uint64(20))
        low = np.flatnonzero(st < np.uint64(RANS_L))
        st[low] = (st[low] << np.uint64(16)) | w[pos[low]]
        pos[low] += 1
        out[:, i] = (e & np.uint64(0xFF)).astype(np.int64) - SYM_OFFSET
    if not np.all(st == np.uint64(RANS_L)):
        raise ValueError("stream did not return to initial state")
    return lane_order_inverse(out, rows, cols, R, C)


def decode_stream_scalar(enc: dict, s: int) -> np.ndarray:
    """Pure-Python decode of one stream (small cases / cross-checks only)."""
    R, C = enc["R"], enc["C"]
    tab = [int(v) for v in enc["table"]]
    w = enc["words"]
    p = int(enc["offs"][s])
    st = (int(w[p]) << 16) | int(w[p + 1])
    p += 2
    res = []
    for _ in range((C // 32) * R):
        e = tab[st & (PROB_M - 1)]
        st = ((e >> 8) & 0xFFF) * (st >> SCALE_BITS) + (e >> 20)
        if st < RANS_L:
            st = (st << 16) | int(w[p])
            p += 1
        res.append((e & 0xFF) - SYM_OFFSET)
    if st != RANS_L:
        raise ValueError("stream did not return to initial state")
    return np.array(res, np.int64)


# -------------------------------------------------------------- reference y
def gemv(codes: np.ndarray, step: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Dequantise-then-matvec in float64: y = (codes * step) @ x."""
    W = np.asarray(codes, np.float64) * np.asarray(step, np.float64)[None, :]
    return W @ np.asarray(x, np.float64)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


# --------------------------------------------------------- synthetic codes
def entropy_bits(codes: np.ndarray) -> float:
    _, c = np.unique(codes, return_counts=True)
    p = c / c.sum()
    return float(-(p * np.log2(p)).sum())


def synth_codes(rows: int, cols: int, target_bits: float, dist: str = "laplace", seed: int = 0):
    """Synthetic ECSQ-like codes (kernel/bench.py:26-35).

    Draw Laplace or standard-normal weights, bisect (40 rounds) the log step
    on [-12, 6] so that the entropy of round(w / step) over the first
    min(rows, 256) rows meets the target, then round and clip to [-127, 127].
    """
    rng = np.random.default_rng(seed)
    if dist == "laplace":
        w = rng.laplace(size=(rows, cols))
    else:
        w = rng.standard_normal((rows, cols))
    lo, hi = -12.0, 6.0
    head = w[: min(rows, 256)]
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if entropy_bits(np.round(head / np.exp(mid))) > target_bits:
            lo = mid
        else:
            hi = mid
    return np.clip(np.round(w / np.exp(0.5 * (lo + hi))), -127, 127).astype(np.int32)


# ------------------------------------------------------------- C oracle
_LIB = None


def c_lib():
    """ctypes handle of the C restatement (oracle/liboracle.so, built by oracle/Makefile)."""
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(path)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        lib.oracle_decode.argtypes = [vp, vp, vp, i32, i32, i32, i32, i64, i64, vp]
        lib.oracle_decode.restype = i64
        lib.oracle_decode_gemv.argtypes = [vp, vp, vp, i32, i32, i32, i32, i64, i64, vp, vp, i32]
        lib.oracle_decode_gemv.restype = i64
        lib.oracle_build_table.argtypes = [vp, i64, vp, vp, vp]
        lib.oracle_build_table.restype = i32
        lib.oracle_encode.argtypes = [vp, i32, i32, i32, i32, vp, vp, vp, i64, vp, vp, i32]
        lib.oracle_encode.restype = i32
        _LIB = lib
    return _LIB


def c_decode(enc: dict, first_stream: int = 0, nstreams: int | None = None) -> np.ndarray:
    """Decode streams [first, first+n) with the C oracle -> int8 (n, R*C/32) in stream order."""
    lib = c_lib()
    rows, cols = enc["shape"]
    R, C = enc["R"], enc["C"]
    words = np.ascontiguousarray(enc["words"], np.uint16)
    offs = np.ascontiguousarray(enc["offs"], np.uint32)
    table = np.ascontiguousarray(enc["table"], np.uint32)
    if nstreams is None:
        nstreams = offs.size - first_stream
    n = (C // 32) * R
    out = np.empty((nstreams, n), np.int8)
    bad = lib.oracle_decode(words.ctypes.data, offs.ctypes.data, table.ctypes.data,
                            rows, cols, R, C, first_stream, nstreams, out.ctypes.data)
    if bad:
        raise ValueError(f"{bad} stream(s) did not return to initial state")
    return out


def c_decode_codes(enc: dict) -> np.ndarray:
    rows, cols = enc["shape"]
    return lane_order_inverse(c_decode(enc).astype(np.int64), rows, cols, enc["R"], enc["C"])


def c_decode_gemv(enc: dict, xs: np.ndarray, first_stream: int = 0,
                  nstreams: int | None = None, threads: int = 1) -> np.ndarray:
    """Fused CPU decode + dot products against pre-scaled x' (float64 accumulate).

    Returns per-stream-row partial sums of shape (rows,) accumulated over the
    requested stream range (rows of other streams are left at 0).
    """
    lib = c_lib()
    rows, cols = enc["shape"]
    R, C = enc["R"], enc["C"]
    words = np.ascontiguousarray(enc["words"], np.uint16)
    offs = np.ascontiguousarray(enc["offs"], np.uint32)
    table = np.ascontiguousarray(enc["table"], np.uint32)
    xs = np.ascontiguousarray(xs, np.float64)
    if nstreams is None:
        nstreams = offs.size - first_stream
    y = np.zeros(rows, np.float64)
    bad = lib.oracle_decode_gemv(words.ctypes.data, offs.ctypes.data, table.ctypes.data,
                                 rows, cols, R, C, first_stream, nstreams,
                                 xs.ctypes.data, y.ctypes.data, threads)
    if bad:
        raise ValueError(f"{bad} stream(s) did not return to initial state")
    return y


def c_build_table(sym: np.ndarray):
    lib = c_lib()
    sym = np.ascontiguousarray(sym, np.uint8).ravel()
    freq = np.zeros(256, np.int64)
    cum = np.zeros(256, np.int64)
    table = np.zeros(PROB_M, np.uint32)
    rc = lib.oracle_build_table(sym.ctypes.data, sym.size, freq.ctypes.data,
                                cum.ctypes.data, table.ctypes.data)
    if rc != 0:
        raise ValueError("degenerate distribution (single symbol)")
    return freq, cum, table


def c_encode(codes: np.ndarray, R: int, C: int, threads: int = 1) -> dict:
    """encode() in C (kernel/rans.py:34-98): same dict, same bytes; OpenMP over
    streams.  For the large shapes of the CPU baseline and bench checks."""
    lib = c_lib()
    codes = np.asarray(codes)
    rows, cols = codes.shape
    check_tiling(rows, cols, R, C)
    sym = codes_to_symbols(codes)
    freq, cum, table = c_build_table(sym)
    c8 = np.ascontiguousarray((sym.astype(np.int16) - SYM_OFFSET).astype(np.int8))
    nstream = rows * cols * 32 // (R * C)
    n = (C // 32) * R
    cap = nstream * (n + 2) + PAD_WORDS
    words = np.empty(cap, np.uint16)
    offs = np.empty(nstream, np.uint32)
    nw = ctypes.c_int64(0)
    rc = lib.oracle_encode(c8.ctypes.data, rows, cols, R, C, freq.ctypes.data, cum.ctypes.data,
                           words.ctypes.data, cap, offs.ctypes.data, ctypes.byref(nw), threads)
    if rc != 0:
        raise RuntimeError(f"oracle_encode failed ({rc})")
    words = words[: nw.value].copy()
    lens_total = nw.value - PAD_WORDS
    nweights = codes.size
    hist = np.bincount(sym.ravel(), minlength=256)
    present = hist > 0
    p = freq[present].astype(np.float64) / PROB_M
    return dict(words=words, offs=offs, table=table, R=R, C=C, shape=tuple(codes.shape),
                bits_payload=16 * (lens_total - 2 * nstream) / nweights,
                bits_state_offs=64 * nstream / nweights,
                bits_table=32 * PROB_M / nweights,
                entropy_model=float(-(hist[present] * np.log2(p)).sum() / nweights))
