"""Benchmark of the fused rANS-decode GEMV over a full decoder step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
                    [--config 2|3] [--bits B] [--layers L]

A "step" is one pass of the hot path over every linear projection of a
decoder step: BASELINE config 2 by default (Qwen2.5-1.5B shapes, 28 layers x
{q,k,v,o,gate,up,down}, discretized-Gaussian codes at 4.25 bits/weight, one
table per matrix, per-column steps 0.01*U[0.5,1.5], bf16 activation N(0,1),
fp32 accumulation).  Weights are synthetic and random (no checkpoints); every
matrix has its own seed.  All 196 projections run from ONE kernel launch
(rans_gemv_step_launch).  The compressed weights (~0.8 GB) exceed the 126 MB
L2, so no flush is needed between steps.

Printed (rank 0, one JSON line): value = effective bf16-equivalent weight
GB/s (2 bytes x weights / step time), ms_per_step, compressed-byte roofline,
the reference CPU path timed on this host (cpu_baseline) and the end-to-end
number through the public API with pinned host buffers (e2e).

--impl reference times the reference's CPU decode path (the oracle port of
kernel/rans.py:101-123 + the dequantise-matvec of kernel/bench.py:54) on the
host cores instead, on the same workload, metric and unit.

N > 1 (torchrun): every projection's output rows are split into contiguous
row-block ranges, one per rank (each rank holds its shard of the encoded
streams, no re-encoding), and each layer's shard outputs are all-gathered over
NCCL after the step kernel.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vram-compression_b200"))

FALLBACK_HBM_GBS = 6650.0   # recipe fallback when MEASURED_PEAKS.json is absent

QWEN15B = [("q", 1536, 1536), ("k", 256, 1536), ("v", 256, 1536), ("o", 1536, 1536),
           ("gate", 8960, 1536), ("up", 8960, 1536), ("down", 1536, 8960)]
QWEN32B = [("q", 5120, 5120), ("k", 1024, 5120), ("v", 1024, 5120), ("o", 5120, 5120),
           ("gate", 27648, 5120), ("up", 27648, 5120), ("down", 5120, 27648)]
LLAMA70B = [("q", 8192, 8192), ("k", 1024, 8192), ("v", 1024, 8192), ("o", 8192, 8192),
            ("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672)]
CONFIGS = {
    # name: (layer shapes, layers, dist, bits, step kind)
    "2": (QWEN15B, 28, "gauss", 4.25, "uniform"),
    "3": (QWEN15B, 28, "laplace", 3.25, "lognormal"),
    "3lo": (QWEN15B, 28, "laplace", 2.25, "lognormal"),
    "4": (QWEN32B, 64, "gauss", 3.25, "uniform"),
    "5": (LLAMA70B, 80, "laplace", 2.25, "lognormal"),
}
MODEL_NAME = {"2": "qwen2.5-1.5b", "3": "qwen2.5-1.5b", "3lo": "qwen2.5-1.5b", "4": "qwen2.5-32b",
              "5": "llama3-70b"}
# configs whose 31-68 G weights are encoded once per distinct layer (see build_workload)
DISTINCT_LAYERS = {"4": 1, "5": 1}
R_TILE = 8


def c_tile(cols: int) -> int:
    """Column-block width: 512 when it divides cols, else the smallest
    multiple of 32 above 512 that does (8960 -> 640)."""
    if cols % 512 == 0:
        return 512
    for c in range(512, cols + 1, 32):
        if cols % c == 0:
            return c
    return cols


# ----------------------------------------------------------------- workload
def scale_for_entropy(dist: str, bits: float) -> float:
    """Step e such that round(w / e) has the target empirical entropy, by the
    bisection of kernel/bench.py:29-33 on a 256 x 1536 sample."""
    rng = np.random.default_rng(12345)
    w = rng.laplace(size=(256, 1536)) if dist == "laplace" else rng.standard_normal((256, 1536))
    lo, hi = -12.0, 6.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        _, c = np.unique(np.round(w / np.exp(mid)), return_counts=True)
        p = c / c.sum()
        if -(p * np.log2(p)).sum() > bits:
            lo = mid
        else:
            hi = mid
    return float(np.exp(0.5 * (lo + hi)))


def make_codes(torch, rows, cols, dist, scale, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    if dist == "laplace":
        u = torch.rand(rows, cols, generator=g, device=device) - 0.5
        w = -torch.sign(u) * torch.log1p(-2 * u.abs())
    else:
        w = torch.randn(rows, cols, generator=g, device=device)
    return torch.clamp(torch.round(w / scale), -127, 127).to(torch.int8).cpu().numpy()


def make_step(cols, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "lognormal":
        return (0.01 * np.exp(rng.normal(0.0, 0.5, cols))).astype(np.float32)
    return (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)


def build_workload(torch, rb, cfg_name, layers, rank, world, device, log, R=None):
    """Encode the step's matrices and place them on the device.

    Configs 4 and 5 (31 G and 68 G weights per step) encode DISTINCT_LAYERS
    layers and copy those encodings into separate device buffers for the
    remaining layers: every layer still has its own weights in HBM (same
    bytes, same traffic), only the CPU encoding time is saved."""
    R = R or R_TILE
    shapes, nlayers, dist, bits, step_kind = CONFIGS[cfg_name]
    nlayers = layers if layers else nlayers
    distinct = DISTINCT_LAYERS.get(cfg_name, nlayers)
    scale = scale_for_entropy(dist, bits)
    nthreads = max(1, len(os.sched_getaffinity(0)))
    mats, meta = [], []
    cache = {}
    t0 = time.time()
    for li in range(nlayers):
        for pi, (name, rows, cols) in enumerate(shapes):
            seed = 1000 * li + pi
            step = make_step(cols, step_kind, seed + 7)
            key = (li % distinct, pi)
            if key not in cache:
                codes = make_codes(torch, rows, cols, dist, scale, 1000 * key[0] + pi, device)
                enc = rb.encode(codes, R, c_tile(cols), nthreads=nthreads)
                del codes
                if li < distinct and li + distinct < nlayers:
                    cache[key] = enc
            else:
                enc = cache[key]
            if world > 1:
                enc, row0, nrows = rb.shard_encoding(enc, rank, world)
            else:
                row0, nrows = 0, rows
            m = rb.RansMatrix(enc, torch.from_numpy(step), device=device)
            mats.append(m)
            meta.append(dict(layer=li, name=name, rows=rows, cols=cols, row0=row0, nrows=nrows,
                             weights=nrows * cols, words=int(enc["words"].size) - rb.PAD_WORDS,
                             nstreams=int(enc["offs"].size), code_entropy=None))
    log(f"encoded {len(mats)} matrices in {time.time() - t0:.1f}s")
    return mats, meta


# ----------------------------------------------------------------- metrics
def algorithmic_bytes(meta):
    """Compressed-byte roofline numerator per step: words (without the 8 pad
    words) + offs + 16 KB table per matrix + bf16 x + fp32 step + fp32 y."""
    b = 0
    for m in meta:
        b += 2 * m["words"] + 4 * m["nstreams"] + 16384 + 2 * m["cols"] + 4 * m["cols"] + 4 * m["nrows"]
    return b


def read_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        try:
            return float(json.load(open(p))["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def read_traffic(workload):
    """dram bytes per launch recorded by the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", f"gemv_step_kernel_{workload}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch"):
            try:
                return float(line.split("=")[1].split()[0])
            except Exception:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []          # (arrival time, fields)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [v.strip() for v in line.split(",")]))

    def stop(self, t0, t1):
        """Summarise the samples that arrived inside the timed window [t0, t1]."""
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.th.join(timeout=2)
        rows = [r for t, r in self.rows if t0 <= t <= t1 + 0.1 and len(r) > 8]
        isnum = lambda v: v.replace(".", "", 1).isdigit()
        sm = [float(r[1]) for r in rows if isnum(r[1])]
        mx = [float(r[2]) for r in rows if isnum(r[2])]
        pw = [float(r[3]) for r in rows if isnum(r[3])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for i, n in enumerate(names):
                if r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU path
def cpu_decode_gemv_sample(mats_host, budget_s, threads):
    """Time the oracle port (C decode + float64 dot, OpenMP over streams) on a
    bounded sample: whole matrices in order until budget_s is spent.
    Returns (weights processed, seconds)."""
    from oracle import rans_oracle as orc
    done_w, spent = 0, 0.0
    while True:
        for enc, xs in mats_host:
            t = time.perf_counter()
            orc.c_decode_gemv(enc, xs, threads=threads)
            spent += time.perf_counter() - t
            done_w += enc["shape"][0] * enc["shape"][1]
            if spent >= budget_s:
                return done_w, spent


def host_sample_matrices(cfg_name, n, seed_base=777):
    """A few matrices of the step's shapes/distribution, generated on the host
    (numpy), with their step-folded activations, for the CPU path."""
    shapes, _, dist, bits, step_kind = CONFIGS[cfg_name]
    import rans_b200 as rb
    scale = scale_for_entropy(dist, bits)
    out = []
    rng = np.random.default_rng(seed_base)
    for i in range(n):
        name, rows, cols = shapes[i % len(shapes)]
        rows = min(rows, 1024)          # the per-weight CPU rate is what is measured
        w = rng.laplace(size=(rows, cols)) if dist == "laplace" else rng.standard_normal((rows, cols))
        codes = np.clip(np.round(w / scale), -127, 127).astype(np.int32)
        enc = rb.encode(codes, R_TILE, c_tile(cols))
        step = make_step(cols, step_kind, seed_base + i)
        x = rng.standard_normal(cols).astype(np.float32)
        out.append((enc, x.astype(np.float64) * step.astype(np.float64)))
    return out


# ----------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--config", default="2", choices=sorted(CONFIGS))
    ap.add_argument("--layers", type=int, default=0, help="override layer count (0 = config's)")
    ap.add_argument("--R", type=int, default=8, choices=[1, 2, 4, 8, 16], help="tile rows of the encoding")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="fused", choices=["fused", "nccl"],
                    help="N>1: outputs written to every rank by the kernel (fused) or NCCL all-gather per layer")
    ap.add_argument("--check", action="store_true", help="N>1: verify the fused exchange against NCCL")
    ap.add_argument("--no-layered", action="store_true", help="skip the dependency-respecting latency number")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    shapes, nl, dist, bits, _ = CONFIGS[args.config]
    nlayers = args.layers or nl
    workload = f"{MODEL_NAME[args.config]}-step-{dist}{bits}".replace(".", "p") + ("" if args.R == 8 else f"-R{args.R}")
    ncores = len(os.sched_getaffinity(0))

    def log(msg):
        if rank == 0:
            print(msg, file=sys.stderr, flush=True)

    weights_full = nlayers * sum(r * c for _, r, c in shapes)

    if args.impl == "reference":
        # the reference's CPU path on this host: rank 0 only
        if rank != 0:
            return
        sample = host_sample_matrices(args.config, len(shapes))
        per_step_budget = 2.0
        for _ in range(args.warmup):
            cpu_decode_gemv_sample(sample[:1], 0.0, ncores)
        w_tot, t_tot = 0, 0.0
        for _ in range(args.steps):
            w, t = cpu_decode_gemv_sample(sample, per_step_budget, ncores)
            w_tot += w
            t_tot += t
        gbs = 2.0 * w_tot / t_tot / 1e9
        ms_step = weights_full / (w_tot / t_tot) * 1e3
        line = {"impl": "reference", "metric": "decode-GEMV effective weight GB/s (bf16-equivalent)",
                "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int32 decode, f64 accumulate",
                "data": "synthetic (seeded numpy codes with the config's shapes and distribution)",
                "config": {"workload": workload, "layers": nlayers, "R": R_TILE, "weights_per_step": weights_full},
                "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": ncores, "kind": "port",
                                 "sample": f"per step: whole {R_TILE}-row-tiled matrices of the step's shapes "
                                           f"until {per_step_budget}s of decode+dot (oracle C port of "
                                           "kernel/rans.py:101-123, OpenMP), extrapolated to a full step"},
                "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import rans_b200 as rb

    if world > 1:
        import datetime
        import torch.distributed as dist_
        torch.cuda.set_device(local)
        dist_.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    else:
        torch.cuda.set_device(0)
    device = torch.device("cuda", torch.cuda.current_device())
    rb.load()

    mats, meta = build_workload(torch, rb, args.config, nlayers, rank, world, device, log, R=args.R)
    # one contiguous activation buffer for the whole step
    xsz = [m.cols for m in mats]
    ysz = [m.rows for m in mats]
    x_all = torch.randn(sum(xsz), generator=torch.Generator(device=device).manual_seed(99),
                        device=device).to(torch.bfloat16)
    xs = list(torch.split(x_all, xsz))
    stream = torch.cuda.current_stream()
    per_layer = len(shapes)
    gather = None
    hdl = None
    if world > 1 and args.exchange == "fused":
        # every rank holds the FULL outputs of every projection in symmetric
        # memory; the kernel stores its shard rows into all ranks' copies
        import rans_dist
        sharded = rans_dist.ShardedStep(mats, [m["rows"] for m in meta], xs, exchange="fused", timeout_ms=60000)
        step, hdl, y_all, F = sharded.step, sharded.hdl, sharded.y_full, sharded.layout.F

        def gather():
            hdl.barrier(channel=0, timeout_ms=60000)
    else:
        y_all = torch.zeros(sum(ysz), device=device)
        ys = list(torch.split(y_all, ysz))
        step = rb.RansStep(mats, xs, ys)
    if world > 1 and args.exchange == "nccl":
        import torch.distributed as dist_
        # per layer: all-gather every rank's shard outputs of the layer's projections
        layer_rows = [sum(ysz[i * per_layer:(i + 1) * per_layer]) for i in range(nlayers)]
        gbufs = [torch.empty(world * max(layer_rows), device=device) for _ in range(nlayers)]
        starts = np.cumsum([0] + ysz)

        def gather():
            for li in range(nlayers):
                a = int(starts[li * per_layer])
                b = int(starts[(li + 1) * per_layer])
                n = b - a
                dist_.all_gather_into_tensor(gbufs[li][: world * n], y_all[a:b])

    def one_step():
        step()
        if gather is not None:
            gather()

    def barrier():
        if world > 1:
            import torch.distributed as dist_
            dist_.barrier()
        torch.cuda.synchronize()

    clk = ClockSampler(torch.cuda.current_device() if world == 1 else local)
    clk.start()
    for _ in range(args.warmup):
        one_step()
    barrier()
    time.sleep(0.5)          # nvidia-smi needs a moment before its first sample
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    # kernel-only timing (same stream as the launches)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    t_wall0 = time.time()
    ev0.record(stream)
    for i in range(args.steps):
        kev[i][0].record(stream)
        step()
        kev[i][1].record(stream)
        if gather is not None:
            gather()
    ev1.record(stream)
    barrier()
    clocks = clk.stop(t_wall0, time.time())
    t_ms = ev0.elapsed_time(ev1) / args.steps
    k_ms = sum(a.elapsed_time(b) for a, b in kev) / args.steps
    if world > 1:
        import torch.distributed as dist_
        tt = torch.tensor([t_ms, k_ms], device=device)
        dist_.all_reduce(tt, op=dist_.ReduceOp.MAX)
        t_ms, k_ms = tt.tolist()

    layered = None
    if world == 1 and not args.no_layered:
        # Dependency-respecting decode: per layer {q,k,v} -> o -> {gate,up} -> down,
        # 4 dependent launches per layer (112 for 28 layers), captured in one
        # CUDA graph.  Same kernels, same inputs; only the ordering differs.
        names = [m["name"] for m in meta]
        phases_of = {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3}
        groups = {}
        for i, (mm, nm) in enumerate(zip(meta, names)):
            groups.setdefault((mm["layer"], phases_of.get(nm, 0)), []).append(i)
        phase_steps = [rb.RansStep([mats[i] for i in idx], [xs[i] for i in idx], [ys[i] for i in idx])
                       for _, idx in sorted(groups.items())]
        for p in phase_steps:
            p()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for p in phase_steps:
                p()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        la, lb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nrep = 20
        la.record(stream)
        for _ in range(nrep):
            g.replay()
        lb.record(stream)
        torch.cuda.synchronize()
        lms = la.elapsed_time(lb) / nrep
        layered = {"us_per_token_step": round(lms * 1e3, 2), "launches_per_step": sum(p.kernels for p in phase_steps),
                   "how": "per layer 4 dependent phases ({q,k,v}, o, {gate,up}, down), one launch each, "
                          "one CUDA graph per step"}
        del g

    exchange_check = None
    if world > 1 and args.check and args.exchange == "fused":
        # same shards through the plain plan, gathered by NCCL, must equal the fused exchange
        import torch.distributed as dist_
        y_plain = torch.zeros(sum(ysz), device=device)
        ref_step = rb.RansStep(mats, xs, list(torch.split(y_plain, ysz)))
        ref_step()
        step()
        gather()
        torch.cuda.synchronize()
        worst = 0.0
        off = 0
        for i, m in enumerate(meta):
            gathered = torch.empty(world * m["nrows"], device=device)
            dist_.all_gather_into_tensor(gathered, y_plain[off: off + m["nrows"]])
            full_i = y_all[int(F[i]): int(F[i]) + m["rows"]]
            worst = max(worst, (gathered - full_i).abs().max().item())
            off += m["nrows"]
        t = torch.tensor([worst], device=device)
        dist_.all_reduce(t, op=dist_.ReduceOp.MAX)
        exchange_check = {"max_abs_diff_vs_nccl_allgather": t.item(), "ok": t.item() == 0.0}

    # end to end through the public API: pinned host x -> device, step, y -> pinned host
    x_host = x_all.cpu().pin_memory()
    y_host = torch.empty(y_all.numel(), dtype=torch.float32).pin_memory()
    for _ in range(args.warmup):
        x_all.copy_(x_host, non_blocking=True)
        one_step()
        y_host.copy_(y_all, non_blocking=True)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        x_all.copy_(x_host, non_blocking=True)
        one_step()
        y_host.copy_(y_all, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        import torch.distributed as dist_
        tt = torch.tensor([e2e_ms], device=device)
        dist_.all_reduce(tt, op=dist_.ReduceOp.MAX)
        e2e_ms = tt.item()

    weights_step = weights_full
    value = 2.0 * weights_step / (t_ms * 1e-3) / 1e9
    e2e_val = 2.0 * weights_step / (e2e_ms * 1e-3) / 1e9
    alg_bytes = algorithmic_bytes(meta)          # this rank's launch
    peak, peak_kind = read_peak()
    achieved = alg_bytes / (k_ms * 1e-3) / 1e9
    traffic = read_traffic(workload) if world == 1 else None
    compressed_gbs_step = alg_bytes * world / (t_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = host_sample_matrices(args.config, len(shapes))
        w, t = cpu_decode_gemv_sample(sample, args.cpu_budget, ncores)
        cpu = {"value": round(2.0 * w / t / 1e9, 3), "unit": "GB/s", "cores": ncores, "kind": "port",
               "sample": f"{w / 1e6:.1f} M weights of the step's shapes/distribution decoded+dotted in "
                         f"{t:.2f}s by the oracle C port of kernel/rans.py:101-123 (OpenMP, {ncores} threads)"}

    if rank == 0:
        line = {
            "metric": "decode-GEMV effective weight GB/s (bf16-equivalent)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms, 4), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "u16 rANS -> f32",
            "data": "synthetic (seeded random codes, steps and bf16 activations; no checkpoint)" +
                    ("" if args.config not in DISTINCT_LAYERS else
                     f"; {DISTINCT_LAYERS[args.config]} distinct encoded layer(s) copied into separate device "
                     f"buffers for all {nlayers} layers"),
            "config": {"workload": workload, "layers": nlayers, "matrices": len(mats), "R": args.R,
                       "C": {str(c): c_tile(c) for c in sorted({c for _, _, c in shapes})},
                       "code_dist": dist, "bits_target": bits, "weights_per_step": weights_step,
                       "compressed_bytes_per_step": alg_bytes * world,
                       "l2": "inputs (compressed weights) larger than the 126 MB L2; no flush",
                       "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
                       "launches_per_step": step.kernels},
            "us_per_token_step": round(t_ms * 1e3, 2),
            "layered": layered,
            "compressed_gbs": round(compressed_gbs_step, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "frac_of_nominal_7700_gbs": round(achieved / 7700.0, 4),
                         "kernel": "gemv_step_kernel", "kernel_ms": round(k_ms, 4)},
            "tsymbols_per_s": round(weights_step / (t_ms * 1e-3) / 1e12, 4),
            "gpu_launches": args.steps * step.kernels,
            "clocks": clocks,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": int(x_all.numel() * 2), "d2h_bytes_per_step": int(y_all.numel() * 4)},
            "cpu_baseline": cpu,
        }
        if world > 1:
            line["exchange"] = {"kind": args.exchange,
                                "how": ("kernel epilogue stores each output row into every rank's output "
                                        "buffer (symmetric memory over NVLink) + one cross-GPU barrier per step"
                                        if args.exchange == "fused" else
                                        "NCCL all_gather_into_tensor per layer after the step kernel"),
                                "check": exchange_check}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist_
        dist_.barrier()
        dist_.destroy_process_group()


if __name__ == "__main__":
    main()
