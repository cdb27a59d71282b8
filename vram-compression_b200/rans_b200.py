"""Host side of the B200 fused rANS-decode GEMV (librans_b200.so).

Mirrors the reference's kernel/rans.py interface so its harness and tests read
the same way:

  build(arch)                 kernel/rans.py:19-30   compile (if stale) + ctypes load
  build_table(sym)            kernel/rans.py:34-51   12-bit static table
  lane_order(sym, R, C)       kernel/rans.py:55-59   tile/lane interleave
  encode(codes, R, C)         kernel/rans.py:62-98   producer (bit-exact, C++)
  RansMatrix(enc, step, lib)  kernel/rans.py:127-162 device-resident matrix
  Int4Matrix(codes, step, lib) kernel/rans.py:165-185 fixed-rate baseline

plus the B200 additions: RansMatrix.gemv_bf16 (step folded into the kernel),
RansStep (every projection of a decoder step from one grid) and RansChain (a
decoder step as a chain of dependent phases from one persistent grid).

There is no CPU fallback: every GEMV/decode goes through librans_b200.so and
raises if the library or a CUDA device is missing.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "librans_b200.so")
SCALE_BITS = 12
M = 1 << SCALE_BITS
RANS_L = 1 << 16
OFFSET = 128
PAD_WORDS = 8
ABI_VERSION = 3

_vp, _i32, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t


class RansGemvDesc(ctypes.Structure):
    """ctypes mirror of the C struct RansGemvDesc (include/rans_b200.h)."""
    _fields_ = [("words", _vp), ("offs", _vp), ("table", _vp), ("x", _vp), ("step", _vp),
                ("y", _vp), ("nwords", _i64), ("rows", ctypes.c_int32), ("cols", ctypes.c_int32),
                ("C", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class RansChainSync(ctypes.Structure):
    """ctypes mirror of the C struct RansChainSync (include/rans_b200.h)."""
    _fields_ = [("nranks", ctypes.c_int32), ("rank", ctypes.c_int32), ("arrive", _vp),
                ("arrive_peer", _vp), ("peer_y", _vp)]


CHAIN_TIMEOUT = -5      # rans_gemv_chain_status: a dependency wait ran out


def _bind(lib):
    # the three reference entry points, with the reference's exact argtypes
    for f in (lib.launch_rans_gemv, lib.launch_rans_decode):
        f.argtypes = [_i32] + [_vp] * 5 + [_i32] * 3 + [_vp]
        f.restype = _i32
    lib.launch_int4_gemv.argtypes = [_vp] * 3 + [_i32] * 2 + [_vp]
    lib.launch_int4_gemv.restype = _i32
    # additive
    lib.rans_gemv_bf16.argtypes = [_i32] + [_vp] * 6 + [_i32] * 3 + [_i64, _vp]
    lib.rans_gemv_bf16.restype = _i32
    lib.rans_gemv_step_workspace_bytes.argtypes = [_vp, _i32, _i32]
    lib.rans_gemv_step_workspace_bytes.restype = _i64
    lib.rans_gemv_step_plan.argtypes = [_vp, _i32, _i32, _vp, _sz, _vp, _vp]
    lib.rans_gemv_step_plan.restype = _i32
    lib.rans_gemv_step_plan_peers.argtypes = [_vp, _vp, _i32, _i32, _i32, _vp, _sz, _vp, _vp]
    lib.rans_gemv_step_plan_peers.restype = _i32
    lib.rans_gemv_step_launch.argtypes = [_i32, _vp, _i32, _vp]
    lib.rans_gemv_step_launch.restype = _i32
    lib.rans_gemv_step_kernels.argtypes = [_vp]
    lib.rans_gemv_step_kernels.restype = _i32
    lib.rans_build_table_host.argtypes = [_vp, _i64, _vp, _vp, _vp, _i32]
    lib.rans_build_table_host.restype = _i32
    lib.rans_encode_bound.argtypes = [_i32] * 4
    lib.rans_encode_bound.restype = _i64
    lib.rans_encode_host.argtypes = [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _vp, _vp, _i32]
    lib.rans_encode_host.restype = _i32
    lib.rans_escape_gemv.argtypes = [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp]
    lib.rans_escape_gemv.restype = _i32
    lib.rans_escape_decode.argtypes = [_vp, _vp, _vp, _i32, _vp, _vp, _i32, _vp]
    lib.rans_escape_decode.restype = _i32
    lib.rans_gemv_chain_workspace_bytes.argtypes = [_vp, _vp, _i32, _i32]
    lib.rans_gemv_chain_workspace_bytes.restype = _i64
    lib.rans_gemv_chain_describe.argtypes = [_vp, _vp, _i32, _i32, _vp, _i64]
    lib.rans_gemv_chain_describe.restype = _i64
    lib.rans_gemv_chain_plan.argtypes = [_vp, _vp, _i32, _i32, _vp, _i32, _vp, _sz, _vp, _vp]
    lib.rans_gemv_chain_plan.restype = _i32
    lib.rans_gemv_chain_launch.argtypes = [_i32, _vp, _i32, _vp]
    lib.rans_gemv_chain_launch.restype = _i32
    lib.rans_gemv_chain_status.argtypes = [_vp, _vp, _vp]
    lib.rans_gemv_chain_status.restype = _i32
    lib.rans_b200_abi_version.argtypes = []
    lib.rans_b200_abi_version.restype = _i32
    return lib


_LIB = None


def build(arch: str = "sm_100a", force: bool = False):
    """Compile librans_b200.so when its sources are newer (nvcc, sm_100a) and load it.

    Same role as the reference's build() (kernel/rans.py:19-30); the returned
    handle also works as the `lib` argument of the reference's own RansMatrix.
    """
    global _LIB
    if arch != "sm_100a":
        raise ValueError("librans_b200 targets sm_100a (B200) only")
    if _LIB is not None and not force:
        return _LIB
    import importlib.util
    spec = importlib.util.spec_from_file_location("rans_b200_build_lib", os.path.join(HERE, "build_lib.py"))
    bl = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bl)
    if force or bl.stale():
        bl.build(force=force)
    if not os.path.exists(LIB):
        raise RuntimeError(f"{LIB} missing and could not be built")
    lib = _bind(ctypes.CDLL(LIB))
    if lib.rans_b200_abi_version() != ABI_VERSION:
        raise RuntimeError("librans_b200.so ABI version mismatch; rebuild it")
    _LIB = lib
    return lib


def load():
    """Load the prebuilt library without trying to compile (GPU box path)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB):
            raise RuntimeError(f"{LIB} missing: run vram-compression_b200/build_lib.py")
        _LIB = _bind(ctypes.CDLL(LIB))
    return _LIB


def _lib(lib=None):
    return lib if lib is not None else (_LIB if _LIB is not None else load())


# --------------------------------------------------------------------- table
def codes_to_int8(codes) -> np.ndarray:
    c = np.asarray(codes)
    if c.size and (int(c.min()) < -OFFSET or int(c.max()) > 255 - OFFSET):
        raise ValueError("code out of 8-bit alphabet (escape not implemented)")
    return np.ascontiguousarray(c.astype(np.int8))


def build_table(sym, nthreads: int = 0):
    """sym: uint8 symbols -> (freq int64[256], cum int64[256], table uint32[4096])."""
    lib = _lib()
    codes = np.ascontiguousarray((np.asarray(sym).astype(np.int16) - OFFSET).astype(np.int8)).ravel()
    table = np.zeros(M, np.uint32)
    freq = np.zeros(256, np.int32)
    cum = np.zeros(256, np.int32)
    rc = lib.rans_build_table_host(codes.ctypes.data, codes.size, table.ctypes.data, freq.ctypes.data,
                                   cum.ctypes.data, nthreads)
    if rc != 0:
        raise AssertionError("degenerate distribution (single symbol)")
    return freq.astype(np.int64), cum.astype(np.int64), table


def table_of_codes(codes, nthreads: int = 0) -> np.ndarray:
    """The 12-bit slot table (uint32[4096]) of integer codes in [-128, 127]
    (kernel/rans.py:34-51), e.g. of a whole matrix whose row ranges are
    encoded separately with encode(..., table=)."""
    lib = _lib()
    c8 = codes_to_int8(codes).ravel()
    table = np.zeros(M, np.uint32)
    freq = np.zeros(256, np.int32)
    cum = np.zeros(256, np.int32)
    if lib.rans_build_table_host(c8.ctypes.data, c8.size, table.ctypes.data, freq.ctypes.data,
                                 cum.ctypes.data, nthreads) != 0:
        raise AssertionError("degenerate distribution (single symbol)")
    return table


# ------------------------------------------------------------------ encoding
def lane_order(sym, R: int, C: int) -> np.ndarray:
    rows, cols = sym.shape
    if not (rows % R == 0 and cols % C == 0 and C % 32 == 0):
        raise AssertionError("rows % R, cols % C and C % 32 must be 0")
    a = sym.reshape(rows // R, R, cols // C, C // 32, 32)
    return a.transpose(0, 2, 4, 3, 1).reshape(-1, (C // 32) * R)


def encode(codes, R: int, C: int, nthreads: int = 0, table=None) -> dict:
    """Encode integer codes in [-128, 127]; returns the reference's dict
    (words uint16, offs uint32, table uint32, R, C, shape, bit accounting).

    table: optional slot table to encode with instead of the one built from
    `codes` -- e.g. the table of a whole matrix when encoding a row-block
    range of it (the streams are then exactly those of the whole matrix's
    encoding; every code must have a non-zero frequency in the table)."""
    lib = _lib()
    codes = np.asarray(codes)
    if codes.ndim != 2:
        raise ValueError("codes must be a 2-D array")
    rows, cols = codes.shape
    if not (rows % R == 0 and cols % C == 0 and C % 32 == 0):
        raise AssertionError("rows % R, cols % C and C % 32 must be 0")
    c8 = codes_to_int8(codes)
    if table is None:
        table = np.zeros(M, np.uint32)
        freq = np.zeros(256, np.int32)
        cum = np.zeros(256, np.int32)
        if lib.rans_build_table_host(c8.ctypes.data, c8.size, table.ctypes.data, freq.ctypes.data,
                                     cum.ctypes.data, nthreads) != 0:
            raise AssertionError("degenerate distribution (single symbol)")
    else:
        table = np.ascontiguousarray(table, np.uint32)
        if table.shape != (M,):
            raise ValueError("table must hold 4096 slots")
        freq = np.bincount((table & 0xFF).astype(np.int64), minlength=256).astype(np.int32)
        present = np.bincount(c8.ravel().astype(np.int16) + OFFSET, minlength=256) > 0
        if np.any(freq[present] == 0):
            raise ValueError("a code has no slot in the given table")
    cap = lib.rans_encode_bound(rows, cols, R, C)
    nstreams = rows * cols * 32 // (R * C)
    words = np.empty(cap, np.uint16)
    offs = np.empty(nstreams, np.uint32)
    nw = ctypes.c_int64(0)
    rc = lib.rans_encode_host(c8.ctypes.data, rows, cols, R, C, table.ctypes.data, words.ctypes.data, cap,
                              offs.ctypes.data, ctypes.byref(nw), nthreads)
    if rc != 0:
        raise RuntimeError(f"rans_encode_host failed ({rc})")
    words = words[: nw.value].copy()
    nweights = codes.size
    lens_total = nw.value - PAD_WORDS
    hist = np.bincount((c8.ravel().astype(np.int16) + OFFSET), minlength=256)
    present = hist > 0
    p = freq[present].astype(np.float64) / M
    entropy_model = float(-(hist[present] * np.log2(p)).sum() / nweights)
    return dict(words=words, offs=offs, table=table, R=R, C=C, shape=codes.shape,
                bits_payload=16 * (lens_total - 2 * nstreams) / nweights,
                bits_state_offs=64 * nstreams / nweights,
                bits_table=32 * M / nweights,
                entropy_model=entropy_model)


def shard_encoding(enc: dict, rank: int, world: int):
    """Rank `rank`'s contiguous row-block range [rb0, rb1) of an encoded matrix,
    as a standalone encoding of shape ((rb1-rb0)*R, cols).

    Streams of consecutive row blocks are consecutive (stream = (rb*ncb+cb)*32
    + lane), so the shard is a slice of offs and of words: no re-encoding.  The
    word slice starts on an 8-word (16-byte) boundary and gets the 8 zero pad
    words a standalone encoding ends with.  Returns (shard, first_row, nrows).
    """
    rows, cols = enc["shape"]
    R, C = enc["R"], enc["C"]
    nrb, ncb = rows // R, cols // C
    rb0, rb1 = nrb * rank // world, nrb * (rank + 1) // world
    s0, s1 = rb0 * ncb * 32, rb1 * ncb * 32
    offs = np.asarray(enc["offs"]).astype(np.int64)
    end = int(np.asarray(enc["words"]).size) - PAD_WORDS
    w0 = int(offs[s0]) if s0 < offs.size else end
    w1 = int(offs[s1]) if s1 < offs.size else end
    w0a = w0 - (w0 % 8)
    words = np.zeros(w1 - w0a + PAD_WORDS, np.uint16)
    words[: w1 - w0a] = np.asarray(enc["words"])[w0a:w1]
    out = dict(enc)
    out.update(words=words, offs=(offs[s0:s1] - w0a).astype(np.uint32), shape=((rb1 - rb0) * R, cols))
    return out, rb0 * R, (rb1 - rb0) * R


# ------------------------------------------------------------------- device
def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("librans_b200 needs a CUDA device (no CPU fallback)")
    return torch


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed with status {rc}")


class RansMatrix:
    """Entropy-coded matrix resident on the GPU (kernel/rans.py:127-162)."""

    def __init__(self, enc, step, lib=None, device=None):
        torch = _torch()
        self.lib = _lib(lib)
        self.R, self.C = enc["R"], enc["C"]
        self.rows, self.cols = enc["shape"]
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        # (np.require copies read-only inputs such as memory-mapped files: torch
        # wraps only writable arrays)
        host = lambda a, t: torch.from_numpy(np.require(a, requirements=["C", "W"]).view(t))
        self.words = host(enc["words"], np.int16).to(dev)
        self.offs = host(enc["offs"], np.int32).to(dev)
        self.table = host(enc["table"], np.int32).to(dev)
        step = step if hasattr(step, "float") else torch.from_numpy(np.asarray(step, np.float32))
        self.step = step.float().to(dev).contiguous()
        self.nwords = int(self.words.numel())
        self.nbytes = sum(t.numel() * t.element_size() for t in (self.words, self.offs, self.table))

    def gemv(self, x, y=None):
        """y = (code * step) @ x via the drop-in entry point (host-side step fold)."""
        torch = _torch()
        xs = (x.float() * self.step).contiguous()
        if y is None:
            y = torch.zeros(self.rows, device=self.device) if self.cols != self.C else \
                torch.empty(self.rows, device=self.device)
        elif self.cols != self.C:
            y.zero_()
        rc = self.lib.launch_rans_gemv(self.R, self.words.data_ptr(), self.offs.data_ptr(),
                                       self.table.data_ptr(), xs.data_ptr(), y.data_ptr(),
                                       self.rows, self.cols, self.C, _stream(torch))
        _check(rc, "launch_rans_gemv")
        return y

    def gemv_bf16(self, x, y=None):
        """y = (code * step) @ x with bf16 x and the step multiplied in-kernel."""
        torch = _torch()
        xb = x.to(torch.bfloat16).contiguous()
        if y is None:
            y = torch.empty(self.rows, device=self.device)
        rc = self.lib.rans_gemv_bf16(self.R, self.words.data_ptr(), self.offs.data_ptr(),
                                     self.table.data_ptr(), xb.data_ptr(), self.step.data_ptr(),
                                     y.data_ptr(), self.rows, self.cols, self.C, self.nwords,
                                     _stream(torch))
        _check(rc, "rans_gemv_bf16")
        return y

    def decode(self, out=None):
        torch = _torch()
        if out is None:
            out = torch.empty(self.rows, self.cols, device=self.device, dtype=torch.bfloat16)
        rc = self.lib.launch_rans_decode(self.R, self.words.data_ptr(), self.offs.data_ptr(),
                                         self.table.data_ptr(), self.step.data_ptr(), out.data_ptr(),
                                         self.rows, self.cols, self.C, _stream(torch))
        _check(rc, "launch_rans_decode")
        return out

    def desc(self, x, y, step=True):
        """RansGemvDesc for the step launcher (x bf16 with step, or fp32 pre-scaled)."""
        return RansGemvDesc(self.words.data_ptr(), self.offs.data_ptr(), self.table.data_ptr(),
                            x.data_ptr(), self.step.data_ptr() if step else None, y.data_ptr(),
                            self.nwords, self.rows, self.cols, self.C, 0)


class Int4Matrix:
    """Fixed-rate 4-bit baseline, codes clipped to [-8, 7] (kernel/rans.py:165-185)."""

    def __init__(self, codes, step, lib=None):
        torch = _torch()
        self.lib = _lib(lib)
        self.rows, self.cols = codes.shape
        q = (np.clip(codes, -8, 7) + 8).astype(np.uint32).reshape(self.rows, -1, 8)
        packed = np.zeros(q.shape[:2], np.uint32)
        for b in range(8):
            packed |= q[:, :, b] << np.uint32(4 * b)
        self.w = torch.from_numpy(packed.view(np.int32)).cuda()
        step = step if hasattr(step, "float") else torch.from_numpy(np.asarray(step, np.float32))
        self.step = step.float().cuda()
        self.nbytes = self.w.numel() * 4

    def gemv(self, x, y=None):
        torch = _torch()
        xs = (x.float() * self.step).contiguous()
        y = torch.empty(self.rows, device="cuda") if y is None else y
        rc = self.lib.launch_int4_gemv(self.w.data_ptr(), xs.data_ptr(), y.data_ptr(), self.rows, self.cols,
                                       _stream(torch))
        _check(rc, "launch_int4_gemv")
        return y


class RansStep:
    """Every projection of a decoder step in one kernel launch.

    `mats` are RansMatrix objects sharing one R; xs are their activations
    (bf16, step folded in-kernel) and ys their fp32 outputs (overwritten).
    The plan is built once; __call__ is one asynchronous launch (of
    `self.kernels` kernels: a large bf16-activation plan adds a prescale).
    """

    def __init__(self, mats, xs, ys, lib=None, peers=None, prescaled_x=False):
        """peers: optional, per matrix the device addresses (valid on this GPU)
        of the matching rows in every rank's output buffer; the kernel then
        writes each output row to all of them (fused all-gather).
        prescaled_x: xs are fp32 activations already multiplied by the step
        (the reference's convention) instead of bf16 with the step applied
        in-kernel."""
        torch = _torch()
        self.lib = _lib(lib)
        if not mats:
            raise ValueError("empty step")
        R = mats[0].R
        if any(m.R != R for m in mats):
            raise ValueError("all matrices of a step must share R")
        self.R = R
        self.mats, self.xs, self.ys = list(mats), list(xs), list(ys)
        arr = (RansGemvDesc * len(mats))(*[m.desc(x, y, step=not prescaled_x) for m, x, y in zip(mats, xs, ys)])
        self._descs = arr
        nbytes = self.lib.rans_gemv_step_workspace_bytes(ctypes.addressof(arr), len(mats), R)
        if nbytes < 0:
            raise ValueError(f"bad step description ({nbytes})")
        self.workspace = torch.empty(int(nbytes), dtype=torch.uint8, device=mats[0].device)
        grid = ctypes.c_int(0)
        if peers is None:
            rc = self.lib.rans_gemv_step_plan(ctypes.addressof(arr), len(mats), R, self.workspace.data_ptr(),
                                              int(nbytes), ctypes.byref(grid), _stream(torch))
            _check(rc, "rans_gemv_step_plan")
        else:
            npeers = len(peers[0])
            if len(peers) != len(mats) or any(len(p) != npeers for p in peers):
                raise ValueError("peers must list the same number of ranks for every matrix")
            flat = (ctypes.c_void_p * (len(mats) * npeers))(*[int(a) for p in peers for a in p])
            self._peer_arr = flat
            rc = self.lib.rans_gemv_step_plan_peers(ctypes.addressof(arr), ctypes.addressof(flat), npeers,
                                                    len(mats), R, self.workspace.data_ptr(), int(nbytes),
                                                    ctypes.byref(grid), _stream(torch))
            _check(rc, "rans_gemv_step_plan_peers")
        self.grid = grid.value
        self.kernels = int(self.lib.rans_gemv_step_kernels(self.workspace.data_ptr()))   # per launch

    def __call__(self):
        torch = _torch()
        rc = self.lib.rans_gemv_step_launch(self.R, self.workspace.data_ptr(), self.grid, _stream(torch))
        _check(rc, "rans_gemv_step_launch")
        return self.ys


class ChainTimeout(RuntimeError):
    """A dependency wait of the chain kernel ran out (the phase it waited for
    never completed in time); that launch's outputs are incomplete."""

    def __init__(self, phase):
        super().__init__(f"chain launch: the wait for phase {phase} ran out")
        self.phase = phase


class RansChain:
    """A decoder step as a chain of dependent phases, from ONE persistent grid.

    mats/xs/ys as for RansStep; phases[i] is matrix i's phase (0..P-1): every
    matrix of phase p+1 starts only when all of phase p is done, so phase
    p+1's x may be phase p's y (mark such matrices in prescaled_x, a bool or
    one flag per matrix: fp32 activations already multiplied by the step;
    the others take bf16 x with the step applied in-kernel).  One call is one
    kernel launch.
    sync: optional (nranks, rank, arrive_ptr, arrive_peer_ptrs, peers) of a
    row-sharded chain over several GPUs (see rans_dist.ShardedChain).
    timeout_ms bounds every wait inside the kernel; check() reports a wait
    that ran out (ChainTimeout).
    """

    def __init__(self, mats, xs, ys, phases, lib=None, prescaled_x=False, timeout_ms=2000, sync=None):
        torch = _torch()
        self.lib = _lib(lib)
        if not mats or len(phases) != len(mats) or len(xs) != len(mats) or len(ys) != len(mats):
            raise ValueError("one activation, output and phase per matrix")
        R = mats[0].R
        if any(m.R != R for m in mats):
            raise ValueError("all matrices of a chain must share R")
        self.R = R
        self.mats, self.xs, self.ys = list(mats), list(xs), list(ys)
        self.phases = [int(p) for p in phases]
        pre = list(prescaled_x) if isinstance(prescaled_x, (list, tuple)) else [bool(prescaled_x)] * len(mats)
        if len(pre) != len(mats):
            raise ValueError("prescaled_x: one flag per matrix")
        arr = (RansGemvDesc * len(mats))(*[m.desc(x, y, step=not p) for m, x, y, p in zip(mats, xs, ys, pre)])
        ph = (ctypes.c_int * len(mats))(*self.phases)
        self._descs, self._ph = arr, ph
        nbytes = self.lib.rans_gemv_chain_workspace_bytes(ctypes.addressof(arr), ctypes.addressof(ph), len(mats), R)
        if nbytes < 0:
            raise ValueError(f"bad chain description ({nbytes})")
        self.workspace = torch.empty(int(nbytes), dtype=torch.uint8, device=mats[0].device)
        sync_p = None
        if sync is not None:
            nranks, rank, arrive, arrive_peer, peers = sync
            if len(arrive_peer) != nranks or len(peers) != len(mats) or any(len(p) != nranks for p in peers):
                raise ValueError("one arrival address per rank and one peer address per rank and matrix")
            self._arrive_peer = (ctypes.c_void_p * nranks)(*[int(a) for a in arrive_peer])
            self._peer_y = (ctypes.c_void_p * (len(mats) * nranks))(*[int(a) for p in peers for a in p])
            self._sync = RansChainSync(nranks, rank, int(arrive), ctypes.addressof(self._arrive_peer),
                                       ctypes.addressof(self._peer_y))
            sync_p = ctypes.addressof(self._sync)
        grid = ctypes.c_int(0)
        rc = self.lib.rans_gemv_chain_plan(ctypes.addressof(arr), ctypes.addressof(ph), len(mats), R, sync_p,
                                           int(timeout_ms), self.workspace.data_ptr(), int(nbytes),
                                           ctypes.byref(grid), _stream(torch))
        _check(rc, "rans_gemv_chain_plan")
        self.grid = grid.value
        self.kernels = 1

    def __call__(self):
        torch = _torch()
        rc = self.lib.rans_gemv_chain_launch(self.R, self.workspace.data_ptr(), self.grid, _stream(torch))
        _check(rc, "rans_gemv_chain_launch")
        return self.ys

    def check(self):
        """Synchronise and raise ChainTimeout if a wait of the launches so far
        ran out (reading it clears it)."""
        torch = _torch()
        phase = ctypes.c_int(-1)
        rc = self.lib.rans_gemv_chain_status(self.workspace.data_ptr(), ctypes.byref(phase), _stream(torch))
        if rc == CHAIN_TIMEOUT:
            raise ChainTimeout(phase.value)
        _check(rc, "rans_gemv_chain_status")
