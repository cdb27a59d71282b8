"""Benchmark of the fused rANS-decode GEMV over a full, dependency-ordered decoder step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
                    [--config 2|3|3lo|4|5] [--layers L] [--R R] [--no-check]

A "step" is one token's pass over every linear projection of a decoder step,
in dependency order: per layer {q,k,v} -> o -> {gate,up} -> down (4 phases per
layer; each phase starts only when the previous one is complete).  Default:
BASELINE config 5, Llama-3-70B shapes, 80 layers x {q,o 8192x8192, k,v
1024x8192, gate,up 28672x8192, down 8192x28672}, discretized Laplacian codes
at 2.25 bits/weight, per-column steps 0.01*exp(N(0,0.5)), bf16 activations
N(0,1), fp32 accumulation.  Weights are synthetic and random (no checkpoints):
one layer's matrices are encoded and copied into separate device buffers for
every layer (every layer has its own ~0.3 GB of compressed weights in HBM,
24 GB in all, far above the 126 MB L2: no flush needed); every layer has its
own steps and activations.

The whole step is ONE launch of the chain kernel (rans_gemv_chain_launch):
a persistent grid that takes chunks in phase order and waits in-kernel for
the previous phase.  N > 1 (torchrun): every projection's output rows are
split into contiguous row-block ranges, one per rank; each rank's kernel
stores its rows of every phase into every rank's full outputs (NVLink,
symmetric memory) and the phase waits for all ranks' arrival signals.

Printed (rank 0, one JSON line): value = effective bf16-equivalent weight
GB/s of the dependent step (2 bytes x weights / step time), ms_per_step,
compressed-byte roofline of the chain kernel, e2e through the public API
(pinned host activations in, outputs out, every step), parity checks of the
timed outputs against the CPU oracle, and (N = 1) the independent-batch
throughput and the one-launch-per-phase graph for comparison.

--impl reference times the reference's CPU path (decode kernel/rans.py:
101-123 + the dequantise-matvec of kernel/bench.py:54, as the oracle's C
port, OpenMP on every host core) on the same workload, metric and unit; it
never loads this repository's library.
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
METRIC = "decode-GEMV effective weight GB/s (bf16-equivalent), dependency-ordered decoder step"

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
PHASE_OF = {"q": 0, "k": 0, "v": 0, "o": 1, "gate": 2, "up": 2, "down": 3}
R_TILE = 8
REL_L2 = 1e-3      # north-star GEMV tolerance
MAX_REL = 1e-4     # kernel/bench.py:55


def c_tile(cols: int) -> int:
    """Column-block width: 512 when it divides cols, else the smallest
    multiple of 32 above 512 that does (8960 -> 640)."""
    if cols % 512 == 0:
        return 512
    for c in range(512, cols + 1, 32):
        if cols % c == 0:
            return c
    return cols


def workload_name(cfg, R):
    _, _, dist, bits, _ = CONFIGS[cfg]
    return f"{MODEL_NAME[cfg]}-step-{dist}{bits}".replace(".", "p") + ("" if R == 8 else f"-R{R}")


def config_dict(cfg, nlayers, R, world, weights):
    shapes, _, dist, bits, step_kind = CONFIGS[cfg]
    d = {"workload": workload_name(cfg, R), "model_shapes": MODEL_NAME[cfg], "layers": nlayers,
         "matrices": nlayers * len(shapes), "R": R,
         "C": {str(c): c_tile(c) for c in sorted({c for _, _, c in shapes})},
         "code_dist": dist, "bits_target": bits, "step_dist": step_kind, "weights_per_step": weights,
         "phases_per_step": 4 * nlayers, "dependency": "per layer {q,k,v} -> o -> {gate,up} -> down",
         "l2": "inputs (compressed weights) larger than the 126 MB L2; no flush",
         "parallelism": f"row-shard x{world}" if world > 1 else "single GPU"}
    return d


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


def make_codes_host(rows, cols, dist, scale, seed):
    """The same distribution drawn with numpy (the reference arm loads no GPU code)."""
    rng = np.random.default_rng(seed)
    w = rng.laplace(size=(rows, cols)) if dist == "laplace" else rng.standard_normal((rows, cols))
    return np.clip(np.round(w / scale), -127, 127).astype(np.int8)


def make_step(cols, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "lognormal":
        return (0.01 * np.exp(rng.normal(0.0, 0.5, cols))).astype(np.float32)
    return (0.01 * rng.uniform(0.5, 1.5, cols)).astype(np.float32)


def build_workload(torch, rb, cfg_name, nlayers, rank, world, device, log, R):
    """Encode the step's matrices (this rank's row shards) and place them on the device.

    Configs 4 and 5 (31 G and 68 G weights per step) encode DISTINCT_LAYERS
    layers and copy those encodings into separate device buffers for the
    remaining layers: every layer still has its own weights in HBM (same
    bytes, same traffic), only the CPU encoding time is saved.  A rank encodes
    only its row-block range, with the table of the whole matrix (the streams
    are exactly those of the whole matrix's encoding).  Returns the matrices,
    their metadata and the host encodings of the distinct layers (for checks)."""
    shapes, _, dist, bits, step_kind = CONFIGS[cfg_name]
    distinct = min(DISTINCT_LAYERS.get(cfg_name, nlayers), nlayers)
    scale = scale_for_entropy(dist, bits)
    nthreads = max(1, len(os.sched_getaffinity(0)) // max(1, world))
    mats, meta, encs = [], [], {}
    t0 = time.time()
    for li in range(nlayers):
        for pi, (name, rows, cols) in enumerate(shapes):
            step = make_step(cols, step_kind, 1000 * li + pi + 7)
            key = (li % distinct, pi)
            if key not in encs:
                codes = make_codes(torch, rows, cols, dist, scale, 1000 * key[0] + pi, device)
                if world > 1:
                    import rans_dist
                    row0, nrows = rans_dist.shard_rows(rows, R, rank, world)
                    table = rb.table_of_codes(codes, nthreads)
                    enc = rb.encode(codes[row0:row0 + nrows], R, c_tile(cols), nthreads=nthreads, table=table)
                else:
                    enc = rb.encode(codes, R, c_tile(cols), nthreads=nthreads)
                del codes
                encs[key] = enc
            enc = encs[key]
            if world > 1:
                import rans_dist
                row0, nrows = rans_dist.shard_rows(rows, R, rank, world)
            else:
                row0, nrows = 0, rows
            m = rb.RansMatrix(enc, torch.from_numpy(step), device=device)
            mats.append(m)
            meta.append(dict(layer=li, name=name, rows=rows, cols=cols, row0=row0, nrows=nrows,
                             weights=nrows * cols, words=int(enc["words"].size) - rb.PAD_WORDS,
                             nstreams=int(enc["offs"].size), key=key, step=step,
                             phase=4 * li + PHASE_OF[name]))
    log(f"encoded and placed {len(mats)} matrices in {time.time() - t0:.1f}s")
    return mats, meta, encs


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
    """dram bytes per launch of the chain kernel over the config's full layer
    count, recorded by the committed ncu summary for this workload, if any."""
    p = os.path.join(ROOT, "profiles", f"gemv_chain_kernel_{workload}.txt")
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
        # nvidia-smi numbers GPUs physically; map through CUDA_VISIBLE_DEVICES
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = vis[gpu_index] if gpu_index < len(vis) else gpu_index
        self.rows = []          # (arrival time, fields)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
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
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.th.join(timeout=2)
        rows = [r for t, r in self.rows if t0 <= t <= t1 + 0.05 and len(r) > 8]
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
def cpu_decode_gemv_sample(sample, budget_s, threads):
    """Time the oracle C port (decode + float64 dot, OpenMP over streams) over
    whole matrices in order until budget_s is spent.  Returns (weights, s)."""
    from oracle import rans_oracle as orc
    done_w, spent = 0, 0.0
    while True:
        for enc, xs in sample:
            t = time.perf_counter()
            orc.c_decode_gemv(enc, xs, threads=threads)
            spent += time.perf_counter() - t
            done_w += enc["shape"][0] * enc["shape"][1]
            if spent >= budget_s:
                return done_w, spent


def decode_ref_scalar_rate(enc, budget_s):
    """Symbols per second of the reference's own per-symbol decode loop
    (kernel/rans.py:101-123, restated by oracle.decode_stream_scalar), one
    core, over evenly spaced streams until budget_s is spent."""
    from oracle import rans_oracle as orc
    n = (enc["C"] // 32) * enc["R"]
    nstreams = enc["offs"].size
    done, spent, i = 0, 0.0, 0
    while spent < budget_s:
        s = (i * 7919) % nstreams
        t = time.perf_counter()
        orc.decode_stream_scalar(enc, s)
        spent += time.perf_counter() - t
        done += n
        i += 1
    return done / spent


def reference_sample(cfg_name, threads, R, seed_base=777):
    """One full layer of the config's shapes (every distinct matrix shape,
    all rows) encoded by the oracle's C restatement of kernel/rans.py:34-98,
    with step-folded activations: the sample the reference arm decodes."""
    from oracle import rans_oracle as orc
    shapes, _, dist, bits, step_kind = CONFIGS[cfg_name]
    scale = scale_for_entropy(dist, bits)
    rng = np.random.default_rng(seed_base)
    out = []
    for i, (name, rows, cols) in enumerate(shapes):
        codes = make_codes_host(rows, cols, dist, scale, seed_base + i)
        enc = orc.c_encode(codes, R, c_tile(cols), threads=threads)
        del codes
        step = make_step(cols, step_kind, seed_base + i)
        x = rng.standard_normal(cols).astype(np.float32)
        out.append((enc, x.astype(np.float64) * step.astype(np.float64)))
    return out


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU path on this host (rank 0 only)."""
    if rank != 0:
        return
    ncores = len(os.sched_getaffinity(0))
    shapes, nl, _, _, _ = CONFIGS[args.config]
    nlayers = args.layers or nl
    weights_full = nlayers * sum(r * c for _, r, c in shapes)
    t0 = time.time()
    sample = reference_sample(args.config, ncores, args.R)
    prep_s = time.time() - t0
    per_step_budget = 2.0
    for _ in range(args.warmup):
        cpu_decode_gemv_sample(sample[1:2], 0.0, ncores)
    w_tot, t_tot = 0, 0.0
    for _ in range(args.steps):
        w, t = cpu_decode_gemv_sample(sample, per_step_budget, ncores)
        w_tot += w
        t_tot += t
    rate = w_tot / t_tot
    gbs = 2.0 * rate / 1e9
    ms_step = weights_full / rate * 1e3
    scalar_rate = decode_ref_scalar_rate(sample[1][0], 2.0)
    layer_w = sum(e["shape"][0] * e["shape"][1] for e, _ in sample)
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "weak" if world == 1 else "strong", "vs_baseline": None,
            "dtype": "int32 decode, f64 accumulate",
            "data": "synthetic (seeded numpy codes with the config's shapes and distribution)",
            "config": config_dict(args.config, nlayers, args.R, world, weights_full),
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": ncores, "kind": "port",
                             "sample": f"per step: whole matrices of one full layer of the step's shapes "
                                       f"({layer_w / 1e6:.0f} M weights, encoded by the oracle's C restatement "
                                       f"of kernel/rans.py:34-98 in {prep_s:.1f}s, untimed), decoded and dotted "
                                       f"in order until {per_step_budget}s (oracle C port of kernel/rans.py:101-123 "
                                       f"+ kernel/bench.py:54, OpenMP, {ncores} threads), extrapolated to a full step"},
            "decode_ref_1core": {"value": round(2.0 * scalar_rate / 1e9, 6), "unit": "GB/s",
                                 "ms_per_step": round(weights_full / scalar_rate * 1e3, 1),
                                 "how": "the reference's per-symbol decode loop (kernel/rans.py:101-123, "
                                        "oracle.decode_stream_scalar) on evenly spaced streams for 2s, one core, "
                                        "extrapolated per symbol to a full step (decode only)"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- checks
def check_outputs(torch, meta, encs, xs, outputs, layers_to_check, world, threads):
    """Timed outputs against the oracle: for the given layers, every matrix's
    rows on this rank (its shard encoding) decoded and dotted in float64 by the
    C oracle.  Returns the worst rel-L2 and max-abs-relative error."""
    from oracle import rans_oracle as orc
    worst_l2, worst_max, nmat = 0.0, 0.0, 0
    for i, m in enumerate(meta):
        if m["layer"] not in layers_to_check:
            continue
        enc = encs[m["key"]]
        x = xs[i].float().cpu().numpy().astype(np.float64)
        yref = orc.c_decode_gemv(enc, x * m["step"].astype(np.float64), threads=threads)
        got = outputs[i].cpu().numpy().astype(np.float64)
        worst_l2 = max(worst_l2, orc.rel_l2(got, yref))
        worst_max = max(worst_max, float(np.abs(got - yref).max() / max(np.abs(yref).max(), 1e-30)))
        nmat += 1
    return worst_l2, worst_max, nmat


# ----------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--config", default="5", choices=sorted(CONFIGS))
    ap.add_argument("--layers", type=int, default=0, help="override layer count (0 = config's)")
    ap.add_argument("--R", type=int, default=8, choices=[1, 2, 4, 8, 16], help="tile rows of the encoding")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the output checks")
    ap.add_argument("--no-compare", action="store_true",
                    help="N=1: skip the independent-batch and one-launch-per-phase comparison timings")
    ap.add_argument("--timeout-ms", type=int, default=5000, help="bound of every in-kernel phase wait")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    shapes, nl, dist, bits, _ = CONFIGS[args.config]
    nlayers = args.layers or nl
    ncores = len(os.sched_getaffinity(0))

    def log(msg):
        if rank == 0:
            print(msg, file=sys.stderr, flush=True)

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
    weights_full = nlayers * sum(r * c for _, r, c in shapes)

    mats, meta, encs = build_workload(torch, rb, args.config, nlayers, rank, world, device, log, args.R)
    phases = [m["phase"] for m in meta]
    xsz = [m.cols for m in mats]
    x_all = torch.randn(sum(xsz), generator=torch.Generator(device=device).manual_seed(99),
                        device=device).to(torch.bfloat16)
    xs = list(torch.split(x_all, xsz))
    stream = torch.cuda.current_stream()

    if world > 1:
        import rans_dist
        import torch.distributed as dist_
        chain = rans_dist.ShardedChain(mats, [m["rows"] for m in meta], xs, phases, timeout_ms=args.timeout_ms)
        outputs = chain.full                         # full outputs on every rank
        local_out = [chain.y_full[a:b] for a, b in chain.layout.local_slices(rank)]
        y_all = chain.y_full
    else:
        y_all = torch.zeros(sum(m.rows for m in mats), device=device)
        outputs = list(torch.split(y_all, [m.rows for m in mats]))
        local_out = outputs
        chain = rb.RansChain(mats, xs, outputs, phases, timeout_ms=args.timeout_ms)

    def barrier():
        if world > 1:
            dist_.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        if world == 1:
            return vals
        t = torch.tensor(vals, device=device, dtype=torch.float64)
        dist_.all_reduce(t, op=dist_.ReduceOp.MAX)
        return t.tolist()

    # ---------------------------------------------------------------- timed
    clk = ClockSampler(torch.cuda.current_device())
    clk.start()
    for _ in range(args.warmup):
        chain()
    chain.check()
    barrier()
    time.sleep(0.3)          # nvidia-smi needs a moment before its first sample
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    t_wall0 = time.time()
    ev0.record(stream)
    for i in range(args.steps):
        kev[i][0].record(stream)
        chain()
        kev[i][1].record(stream)
    ev1.record(stream)
    barrier()
    clocks = clk.stop(t_wall0, time.time())
    chain.check()
    t_ms = ev0.elapsed_time(ev1) / args.steps
    k_ms = sum(a.elapsed_time(b) for a, b in kev) / args.steps
    t_ms, k_ms = max_over_ranks([t_ms, k_ms])

    # ---------------------------------------------------------------- checks
    check = None
    if not args.no_check:
        # the timed launch's outputs (the last one) against the C oracle:
        # first and last layer (every distinct shape, two device copies)
        torch.cuda.synchronize()
        lay = sorted({0, nlayers - 1})
        l2, mx, nmat = check_outputs(torch, meta, encs, xs, local_out, lay, world, max(1, ncores // world))
        l2, mx = max_over_ranks([l2, mx])
        check = {"layers": lay, "matrices_per_rank": nmat, "max_rel_l2": l2, "max_abs_rel": mx,
                 "tolerance": {"rel_l2": REL_L2, "max_abs_rel": MAX_REL},
                 "ok": bool(l2 <= REL_L2 and mx < MAX_REL),
                 "how": "chain outputs of the last timed launch vs float64 decode+dot of the same encoding "
                        "(oracle C restatement of kernel/rans.py:101-123 + kernel/bench.py:54)"}
        if world > 1:
            # the exchange: every rank holds the same full outputs
            hi = y_all.clone()
            lo = y_all.clone()
            dist_.all_reduce(hi, op=dist_.ReduceOp.MAX)
            dist_.all_reduce(lo, op=dist_.ReduceOp.MIN)
            same = bool(torch.equal(hi, y_all) and torch.equal(lo, y_all))
            same = bool(max_over_ranks([0.0 if same else 1.0])[0] == 0.0)
            check["exchange_identical_on_all_ranks"] = same
            check["ok"] = check["ok"] and same
        log(f"check: {check}")

    compare = None
    if world == 1 and not args.no_compare:
        # the same projections as an independent batch (one step launch) and
        # as one launch per phase (CUDA graph): throughput and launch-gap context
        ys_b = [torch.empty(m.rows, device=device) for m in mats]
        batch = rb.RansStep(mats, xs, ys_b)
        for _ in range(3):
            batch()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            batch()
        b.record(stream)
        torch.cuda.synchronize()
        batch_ms = a.elapsed_time(b) / args.steps
        ys_p = [torch.empty(m.rows, device=device) for m in mats]
        groups = {}
        for i, p in enumerate(phases):
            groups.setdefault(p, []).append(i)
        per_phase = [rb.RansStep([mats[i] for i in idx], [xs[i] for i in idx], [ys_p[i] for i in idx])
                     for _, idx in sorted(groups.items())]
        for p in per_phase:
            p()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for p in per_phase:
                p()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(args.steps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        graph_ms = a.elapsed_time(b) / args.steps
        chain()
        torch.cuda.synchronize()
        # the chain decodes the last wave of a multi-wave phase with half-size
        # items (another summation order), so compare within fp32 rounding
        diff = max(float((u - v).norm() / v.norm().clamp_min(1e-30)) for u, v in zip(outputs, ys_p))
        compare = {"independent_batch": {"us_per_step": round(batch_ms * 1e3, 1),
                                         "gbs": round(2.0 * weights_full / (batch_ms * 1e-3) / 1e9, 1),
                                         "compressed_gbs": round(algorithmic_bytes(meta) / (batch_ms * 1e-3) / 1e9, 1),
                                         "roofline_frac": round(algorithmic_bytes(meta) / (batch_ms * 1e-3) / 1e9
                                                                / read_peak()[0], 4),
                                         "how": "all projections as one independent batch "
                                                "(rans_gemv_step_launch; ignores the phase order)"},
                   "per_phase_graph": {"us_per_step": round(graph_ms * 1e3, 1),
                                       "launches_per_step": sum(p.kernels for p in per_phase),
                                       "max_rel_l2_vs_chain": diff,
                                       "how": "one step launch per phase, captured in one CUDA graph"},
                   "chain_over_batch": round(t_ms / batch_ms, 3)}
        del g
        if check is not None:
            check["chain_vs_per_phase_launches_max_rel_l2"] = diff
            check["ok"] = check["ok"] and diff <= 1e-6

    # ---------------------------------------------------------------- e2e
    # through the public API: this step's activations from pinned host memory,
    # the chain launch, and this rank's output rows back to pinned host memory
    x_host = x_all.cpu().pin_memory()
    if world > 1:
        # this rank's rows of every projection, gathered into one buffer
        idx = torch.cat([torch.arange(a, b, device=device) for a, b in chain.layout.local_slices(rank)])
        y_src = torch.empty(idx.numel(), device=device)
    else:
        idx, y_src = None, y_all
    y_host = torch.empty(y_src.numel(), dtype=torch.float32).pin_memory()

    def e2e_step():
        x_all.copy_(x_host, non_blocking=True)
        chain()
        if idx is not None:
            torch.index_select(y_all, 0, idx, out=y_src)
        y_host.copy_(y_src, non_blocking=True)

    d2h_bytes = 4 * y_src.numel()
    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    chain.check()
    e2e_ms = max_over_ranks([e0.elapsed_time(e1) / args.steps])[0]

    # ---------------------------------------------------------------- report
    value = 2.0 * weights_full / (t_ms * 1e-3) / 1e9
    e2e_val = 2.0 * weights_full / (e2e_ms * 1e-3) / 1e9
    alg_bytes = algorithmic_bytes(meta)          # this rank's launch
    peak, peak_kind = read_peak()
    achieved = alg_bytes / (k_ms * 1e-3) / 1e9
    traffic = read_traffic(workload_name(args.config, args.R)) if world == 1 else None
    if traffic is not None:
        traffic *= nlayers / nl   # the summary's figure is for the config's full layer count
    compressed_total = alg_bytes
    if world > 1:
        t_b = torch.tensor([float(alg_bytes)], device=device, dtype=torch.float64)
        dist_.all_reduce(t_b)
        compressed_total = int(t_b.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = []
        for pi, (name, rows, cols) in enumerate(shapes):
            enc = encs[(0, pi)]
            m = meta[pi]
            sample.append((enc, xs[pi].float().cpu().numpy().astype(np.float64) * m["step"].astype(np.float64)))
        w, t = cpu_decode_gemv_sample(sample, args.cpu_budget, ncores)
        cpu = {"value": round(2.0 * w / t / 1e9, 3), "unit": "GB/s", "cores": ncores, "kind": "port",
               "sample": f"{w / 1e6:.1f} M weights (whole matrices of layer 0, in order) decoded and dotted in "
                         f"{t:.2f}s by the oracle C port of kernel/rans.py:101-123 (OpenMP, {ncores} threads)"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms, 4), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "u16 rANS -> f32",
            "data": "synthetic (seeded random codes, steps and bf16 activations; no checkpoint)" +
                    ("" if args.config not in DISTINCT_LAYERS else
                     f"; {DISTINCT_LAYERS[args.config]} distinct encoded layer copied into separate device "
                     f"buffers for all {nlayers} layers"),
            "config": config_dict(args.config, nlayers, args.R, world, weights_full),
            "compressed_bytes_per_step": compressed_total,
            "us_per_token_step": round(t_ms * 1e3, 2),
            "launches_per_step": 1,
            "compressed_gbs": round(compressed_total / (t_ms * 1e-3) / 1e9, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "frac_of_nominal_7700_gbs": round(achieved / 7700.0, 4),
                         "kernel": "gemv_chain_kernel", "kernel_ms": round(k_ms, 4),
                         "per": "rank" if world > 1 else "gpu"},
            "tsymbols_per_s": round(weights_full / (t_ms * 1e-3) / 1e12, 4),
            "gpu_launches": args.steps,
            "clocks": clocks,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": int(x_all.numel() * 2), "d2h_bytes_per_step": int(d2h_bytes),
                    "how": "per step: all activations H2D from pinned memory, one chain launch, this rank's "
                           "output rows D2H to pinned memory (max over ranks)"},
            "check": check,
            "compare": compare,
            "cpu_baseline": cpu,
        }
        if world > 1:
            line["exchange"] = {"kind": "fused",
                                "how": "each phase's output rows stored by the kernel into every rank's full "
                                       "outputs (symmetric memory over NVLink), then an in-kernel wait per phase "
                                       "for every rank's arrival signal"}
        print(json.dumps(line), flush=True)
    if world > 1:
        chain.close()
        dist_.barrier()
        dist_.destroy_process_group()


if __name__ == "__main__":
    main()
