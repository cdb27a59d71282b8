"""Model integration on top of librans_b200: quantised codes -> escape split ->
rANS encoding -> an on-disk container -> a GPU linear layer.

The reference stops at the kernel: its quantisers (exp/quant.py) produce
integer codes and per-column steps, its encoder (kernel/rans.py:62-98) takes
codes in [-128, 127] only, and "escape codes, model integration" are listed as
next steps in its README.  This module connects the two ends:

  entropy_bits(codes)            exp/quant.py:22-25   zero-order entropy of codes
  ecsq_rtn(W, bits, base)        exp/quant.py:122-146 entropy-targeted uniform grid
                                                      (the RTN bisection; the GPTQ
                                                      refinement needs calibration
                                                      Hessians and stays upstream)
  split_escapes(codes)           codes outside [-128, 127] -> fill code + side list
  EncodedMatrix.encode(...)      rans_b200.encode (bit-exact with kernel/rans.py)
  save_matrices / load_matrices  one-file container, 64-byte aligned arrays, mmap
  RansLinear                     torch module: batch-1 fused decode-GEMV (bf16 x,
                                 step in-kernel), larger batches decode to bf16
                                 and use a dense GEMM; escapes completed by
                                 rans_escape_gemv / rans_escape_decode

Everything that touches the GPU goes through librans_b200.so; there is no CPU
fallback.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field

import numpy as np

import rans_b200 as rb

ALPHABET_LO, ALPHABET_HI = -128, 127
MAGIC = b"RANSB200"
FORMAT = "rans-b200-matrices"
FORMAT_VERSION = 1
ALIGN = 64


# ------------------------------------------------------------- quantisation
def entropy_bits(codes) -> float:
    """Empirical zero-order entropy in bits per code (exp/quant.py:22-25)."""
    c = np.asarray(codes).ravel()
    if c.size == 0:
        return 0.0
    c = c.astype(np.int64)
    counts = np.bincount(c - c.min())
    p = counts[counts > 0].astype(np.float64) / c.size
    return float(-(p * np.log2(p)).sum())


def ecsq_rtn(W, target_bits: float, base=None, iters: int = 40):
    """Entropy-constrained uniform quantisation, round-to-nearest.

    Step per input column = exp(logc) * base[col] (base = 1 without
    waterfilling); logc is bisected for `iters` rounds so that the entropy of
    round(W / step) meets `target_bits` (entropy falls as the step grows), over
    the same bracket as exp/quant.py:139-146.  Returns (codes int32, step
    float32[cols]).  Codes are unbounded: values outside [-128, 127] become
    escapes in EncodedMatrix.encode.
    """
    W = np.asarray(W, np.float64)
    if W.ndim != 2:
        raise ValueError("W must be 2-D (out_features x in_features)")
    b = np.ones(W.shape[1]) if base is None else np.asarray(base, np.float64)
    std = float(W.std())
    if not std > 0:
        raise ValueError("W is constant")
    lo, hi = math.log(std) - 12, math.log(std) + 4

    def h(logc):
        return entropy_bits(np.rint(W / (math.exp(logc) * b)))

    for _ in range(iters):
        mid = (lo + hi) / 2
        if h(mid) > target_bits:
            lo = mid
        else:
            hi = mid
    step = (math.exp((lo + hi) / 2) * b).astype(np.float32)
    codes = np.rint(W / step.astype(np.float64)).astype(np.int64)
    if np.abs(codes).max() >= 2 ** 31:
        raise ValueError("codes overflow int32")
    return codes.astype(np.int32), step


# -------------------------------------------------------------------- escapes
def split_escapes(codes, fill=None):
    """Codes outside [-128, 127] -> (in-range int8 codes, rows, cols, codes, fill).

    Out-of-range positions take `fill` in the stream (default: the most
    frequent in-range code, so an escape costs the stream the fewest bits) and
    are listed exactly in (rows, cols, codes), int32, row-major order.
    """
    c = np.asarray(codes)
    if c.ndim != 2:
        raise ValueError("codes must be 2-D")
    c = c.astype(np.int64)
    out = (c < ALPHABET_LO) | (c > ALPHABET_HI)
    if fill is None:
        inr = c[~out]
        if inr.size:
            hist = np.bincount(inr - ALPHABET_LO, minlength=256)
            fill = int(np.argmax(hist)) + ALPHABET_LO
        else:
            fill = 0
    if not ALPHABET_LO <= fill <= ALPHABET_HI:
        raise ValueError("fill code must be in [-128, 127]")
    r, k = np.nonzero(out)
    esc_codes = c[r, k]
    if esc_codes.size and np.abs(esc_codes).max() >= 2 ** 31:
        raise ValueError("escape codes overflow int32")
    c8 = np.where(out, fill, c).astype(np.int8)
    return c8, r.astype(np.int32), k.astype(np.int32), esc_codes.astype(np.int32), int(fill)


def merge_escapes(c8, rows, cols, codes):
    """Inverse of split_escapes: the full int32 code matrix."""
    full = np.asarray(c8).astype(np.int32).copy()
    full[np.asarray(rows, np.int64), np.asarray(cols, np.int64)] = np.asarray(codes, np.int32)
    return full


# ---------------------------------------------------------- encoded matrices
@dataclass
class EncodedMatrix:
    """Host-side encoded matrix: the reference's encoding dict (words, offs,
    table, R, C, shape) plus per-column steps and the escape list."""
    enc: dict
    step: np.ndarray
    esc_rows: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    esc_cols: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    esc_codes: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int32))
    fill: int = 0

    @property
    def shape(self):
        return tuple(self.enc["shape"])

    @property
    def n_escapes(self) -> int:
        return int(self.esc_rows.size)

    @classmethod
    def encode(cls, codes, step, R: int = 8, C: int = 512, nthreads: int = 0):
        c8, er, ec, eco, fill = split_escapes(codes)
        enc = rb.encode(c8, R, C, nthreads=nthreads)
        step = np.ascontiguousarray(np.asarray(step, np.float32))
        if step.shape != (c8.shape[1],):
            raise ValueError("step must have one entry per column")
        return cls(enc, step, er, ec, eco, fill)

    def nbytes(self) -> int:
        """Stored bytes: stream words, offs, table, steps and escapes."""
        return int(sum(np.asarray(a).nbytes for a in (self.enc["words"], self.enc["offs"], self.enc["table"],
                                                        self.step, self.esc_rows, self.esc_cols, self.esc_codes)))

    def bits_per_weight(self) -> float:
        rows, cols = self.shape
        return 8.0 * self.nbytes() / (rows * cols)


# ------------------------------------------------------------ file container
# Layout: MAGIC (8 bytes) | uint64 LE header length | UTF-8 JSON header |
# zero padding to a 64-byte boundary | data region.  Every array starts at a
# 64-byte aligned offset of the data region (offsets in the header are
# relative to it), little-endian, C order, so a file can be memory-mapped and
# each array viewed without copies.
_ARRAYS = (("words", "<u2"), ("offs", "<u4"), ("table", "<u4"), ("step", "<f4"),
           ("esc_rows", "<i4"), ("esc_cols", "<i4"), ("esc_codes", "<i4"))


def _arrays_of(m: EncodedMatrix):
    return {"words": m.enc["words"], "offs": m.enc["offs"], "table": m.enc["table"], "step": m.step,
            "esc_rows": m.esc_rows, "esc_cols": m.esc_cols, "esc_codes": m.esc_codes}


def save_matrices(path: str, mats: dict, meta: dict | None = None) -> None:
    """Write {name: EncodedMatrix} to one file (see the layout above)."""
    entries, blobs, off = {}, [], 0
    for name, m in mats.items():
        arrs = {}
        for key, dt in _ARRAYS:
            a = np.ascontiguousarray(np.asarray(_arrays_of(m)[key]).astype(dt, copy=False))
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            arrs[key] = {"dtype": dt, "offset": off, "count": int(a.size)}
            blobs.append((off, a))
            off += a.nbytes
        rows, cols = m.shape
        bits = {k: float(m.enc[k]) for k in ("bits_payload", "bits_state_offs", "bits_table", "entropy_model")
                if k in m.enc}
        entries[name] = {"rows": int(rows), "cols": int(cols), "R": int(m.enc["R"]), "C": int(m.enc["C"]),
                         "fill": int(m.fill), "arrays": arrs, "bits": bits}
    header = json.dumps({"format": FORMAT, "version": FORMAT_VERSION, "matrices": entries,
                         "meta": meta or {}}, sort_keys=True).encode()
    start = (16 + len(header) + ALIGN - 1) // ALIGN * ALIGN
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(np.uint64(len(header)).tobytes())
        f.write(header)
        f.write(b"\0" * (start - 16 - len(header)))
        pos = start
        for o, a in blobs:
            f.write(b"\0" * (start + o - pos))
            f.write(a.tobytes())
            pos = start + o + a.nbytes
    os.replace(tmp, path)


def load_matrices(path: str, mmap: bool = True):
    """Read a container: returns ({name: EncodedMatrix}, meta).  With mmap the
    arrays are read-only views of the mapped file."""
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path}: not a {FORMAT} file")
        hlen = int(np.frombuffer(f.read(8), "<u8")[0])
        header = json.loads(f.read(hlen).decode())
    if header.get("format") != FORMAT or header.get("version") != FORMAT_VERSION:
        raise ValueError(f"{path}: unsupported format {header.get('format')} v{header.get('version')}")
    start = (16 + hlen + ALIGN - 1) // ALIGN * ALIGN
    buf = np.memmap(path, dtype=np.uint8, mode="r") if mmap else np.fromfile(path, dtype=np.uint8)
    out = {}
    for name, e in header["matrices"].items():
        arrs = {}
        for key, dt in _ARRAYS:
            a = e["arrays"][key]
            nbytes = a["count"] * np.dtype(dt).itemsize
            lo = start + a["offset"]
            if lo + nbytes > buf.size:
                raise ValueError(f"{path}: array {name}.{key} past the end of the file")
            arrs[key] = buf[lo:lo + nbytes].view(dt)
        enc = dict(words=arrs["words"], offs=arrs["offs"], table=arrs["table"], R=e["R"], C=e["C"],
                   shape=(e["rows"], e["cols"]), **e.get("bits", {}))
        out[name] = EncodedMatrix(enc, arrs["step"], arrs["esc_rows"], arrs["esc_cols"], arrs["esc_codes"],
                                  e["fill"])
    return out, header.get("meta", {})


# -------------------------------------------------------------- torch layer
def _torch_nn():
    import torch
    return torch


class RansLinear(_torch_nn().nn.Module):
    """y = x @ W^T (+ bias) with W = code * step kept entropy coded on the GPU.

    One input row (batch-1 decode): the fused decode-GEMV with bf16 x and the
    step applied in-kernel (rans_gemv_bf16), then rans_escape_gemv.  More rows:
    the matrix is decoded to a transient bf16 copy (launch_rans_decode +
    rans_escape_decode) and multiplied densely.
    """

    def __init__(self, m: EncodedMatrix, bias=None, lib=None, device=None):
        super().__init__()
        torch = rb._torch()
        self.mat = rb.RansMatrix(m.enc, torch.from_numpy(np.array(m.step, np.float32)), lib=lib, device=device)
        dev = self.mat.device
        self.out_features, self.in_features = m.shape
        self.n_escapes = m.n_escapes
        self.fill = m.fill
        self.esc_rows = torch.from_numpy(np.array(m.esc_rows, np.int32)).to(dev)
        self.esc_cols = torch.from_numpy(np.array(m.esc_cols, np.int32)).to(dev)
        self.esc_codes = torch.from_numpy(np.array(m.esc_codes, np.int32)).to(dev)
        self.esc_delta = (self.esc_codes.double() - float(m.fill)).float()
        self.bias = None if bias is None else torch.as_tensor(bias).float().to(dev)
        self.stored_bytes = m.nbytes()

    @classmethod
    def from_weight(cls, weight, bits: float, bias=None, R: int = 8, C: int = 512, base=None, lib=None):
        """Quantise a dense weight (out x in) with ecsq_rtn at `bits` and encode it."""
        w = weight.detach().float().cpu().numpy() if hasattr(weight, "detach") else np.asarray(weight)
        codes, step = ecsq_rtn(w, bits, base)
        return cls(EncodedMatrix.encode(codes, step, R, C), bias=bias, lib=lib)

    def gemv(self, x, y=None):
        """One activation vector (in_features) -> fp32 y (out_features)."""
        torch = rb._torch()
        m = self.mat
        xb = x.reshape(-1).to(torch.bfloat16).contiguous()
        if y is None:
            y = torch.empty(m.rows, device=m.device)
        st = rb._stream(torch)
        rb._check(m.lib.rans_gemv_bf16(m.R, m.words.data_ptr(), m.offs.data_ptr(), m.table.data_ptr(),
                                       xb.data_ptr(), m.step.data_ptr(), y.data_ptr(), m.rows, m.cols, m.C,
                                       m.nwords, st), "rans_gemv_bf16")
        if self.n_escapes:
            rb._check(m.lib.rans_escape_gemv(self.esc_rows.data_ptr(), self.esc_cols.data_ptr(),
                                             self.esc_delta.data_ptr(), self.n_escapes, xb.data_ptr(),
                                             m.step.data_ptr(), y.data_ptr(), st), "rans_escape_gemv")
        return y

    def weight_bf16(self, out=None):
        """The dense bf16 weight bf16(code * step), escapes included."""
        torch = rb._torch()
        m = self.mat
        out = m.decode(out)
        if self.n_escapes:
            rb._check(m.lib.rans_escape_decode(self.esc_rows.data_ptr(), self.esc_cols.data_ptr(),
                                               self.esc_codes.data_ptr(), self.n_escapes, m.step.data_ptr(),
                                               out.data_ptr(), m.cols, rb._stream(torch)), "rans_escape_decode")
        return out

    def forward(self, x):
        torch = rb._torch()
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected last dim {self.in_features}, got {x.shape[-1]}")
        lead = x.shape[:-1]
        n = int(np.prod(lead)) if len(lead) else 1
        if n == 1:
            y = self.gemv(x)
            if self.bias is not None:
                y = y + self.bias
            return y.to(x.dtype).reshape(*lead, self.out_features)
        w = self.weight_bf16()
        y = torch.nn.functional.linear(x.reshape(n, -1).to(torch.bfloat16), w).float()
        if self.bias is not None:
            y = y + self.bias
        return y.to(x.dtype).reshape(*lead, self.out_features)
