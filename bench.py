#!/usr/bin/env python
"""Benchmark: trees/sec on BASELINE config 2 (Logloss, 10M x 200 float32 features,
half N(0,1) / half U(0,1), 5% NaN, border_count 128 (nan_mode=Min sentinel),
depth 8, lr 0.05, Bayesian bootstrap T=1, Cosine score, l2 3), plus the
histogram kernel's achieved HBM bandwidth against the measured peak.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --config 3|4 [--variant ...]   (bench_configs.py: MultiClass / ranking)

A step is one boosting iteration (one tree).  Multi-GPU runs are launched by
torchrun, one rank per GPU; rows are document-sharded (strong scaling: the
10M-row job is split across the ranks) and every level's histograms are summed
with NCCL.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BLOCK_ROWS = 1 << 20       # data is generated in fixed 1Mi-row blocks so any sharding sees the same rows
# cb-train hands the seam the learning rate narrowed to f32 (boosting.rs:4958)
LR_SEAM = float(np.float32(0.05))
BORDER_SAMPLE = 200_000    # fixed-seed sample the borders are selected from (cf. cb-data's 200k sample)
FMIN = float(np.finfo(np.float32).min)
# DRAM bytes (read + write) per histogrammed row of the histogram kernel, from
# an ncu capture of the eight histogram launches of one config-2-shaped tree at
# 2M rows, kept with the profiles; the roofline's `traffic` scales it by the
# rows each launch histograms.
HIST_DRAM_CAPTURE = os.path.join(ROOT, "profiles", "hist_kernel_dram_2M.json")


def hist_dram_bytes_per_row():
    try:
        with open(HIST_DRAM_CAPTURE) as f:
            d = json.load(f)
        return float(d["dram_bytes_per_hist_row"]), d["command"]
    except Exception:
        return None, None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# synthetic data (config 2 shapes and distributions; no public dataset exists)
# ---------------------------------------------------------------------------

def _block(b: int, F: int, seed: int):
    """Rows [b*BLOCK_ROWS, (b+1)*BLOCK_ROWS): features [F][rows] f32 and label."""
    g = np.random.default_rng([seed, b])
    m = BLOCK_ROWS
    X = np.empty((F, m), dtype=np.float32)
    h = F // 2
    X[:h] = g.standard_normal((h, m), dtype=np.float32)
    X[h:] = g.random((F - h, m), dtype=np.float32)
    nan = g.random((F, m), dtype=np.float32) < 0.05
    X[nan] = np.nan
    # label ~ Bernoulli(sigmoid(sparse linear over 20 features + pairwise terms))
    gw = np.random.default_rng([seed, 1 << 30])
    k = min(20, F)
    feats = gw.choice(F, size=k, replace=False)
    coef = gw.standard_normal(k)
    pairs = gw.choice(k, size=(10, 2))
    pcoef = gw.standard_normal(10) * 0.5
    Z = np.nan_to_num(X[feats].astype(np.float64))
    z = coef @ Z
    for (i, j), c in zip(pairs, pcoef):
        z += c * Z[i] * Z[j]
    y = (g.random(m) < 1.0 / (1.0 + np.exp(-z))).astype(np.float64)
    return X, y


def make_shard(row_offset: int, n: int, F: int, seed: int, block=None):
    """Rows [row_offset, row_offset + n) as features [F][n] f32 and labels; the
    1Mi-row blocks are generated on a thread pool (each block has its own
    seeded generator, so the rows do not depend on the thread count).  block:
    the per-block generator (config 2's by default)."""
    block = block or _block
    from concurrent.futures import ThreadPoolExecutor
    X = np.empty((F, n), dtype=np.float32)
    y = np.empty(n, dtype=np.float64)
    b0, b1 = row_offset // BLOCK_ROWS, (row_offset + n - 1) // BLOCK_ROWS

    def fill(b):
        Xb, yb = block(b, F, seed)
        lo = max(row_offset, b * BLOCK_ROWS)
        hi = min(row_offset + n, (b + 1) * BLOCK_ROWS)
        X[:, lo - row_offset:hi - row_offset] = Xb[:, lo - b * BLOCK_ROWS:hi - b * BLOCK_ROWS]
        y[lo - row_offset:hi - row_offset] = yb[lo - b * BLOCK_ROWS:hi - b * BLOCK_ROWS]

    if n > 0:
        # each worker holds one F x 1Mi block: share the host cores among the
        # ranks of a box so their blocks fit in host memory together
        per_rank = max(1, (os.cpu_count() or 1) // max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1"))))
        workers = max(1, min(b1 - b0 + 1, per_rank, 16))
        with ThreadPoolExecutor(workers) as ex:
            list(ex.map(fill, range(b0, b1 + 1)))
    return X, y


def _block5(b: int, F: int, seed: int):
    """Config 5 rows: F N(0,1) f32 features, target = a sparse linear score over
    25 features plus N(0, 0.1) noise (RMSE)."""
    g = np.random.default_rng([seed, b, 5])
    X = g.standard_normal((F, BLOCK_ROWS), dtype=np.float32)
    gw = np.random.default_rng([seed, 1 << 30, 5])
    k = min(25, F)
    feats = gw.choice(F, size=k, replace=False)
    y = gw.standard_normal(k) @ X[feats].astype(np.float64) + 0.1 * g.standard_normal(BLOCK_ROWS)
    return X, y


def make_borders5(F: int, border_count: int, seed: int):
    """Uniform-quantile borders of config 5's N(0,1) features from a fixed-seed
    200k sample (no NaN, so no sentinel)."""
    g = np.random.default_rng([seed, 1 << 31, 5])
    out = []
    for _ in range(F):
        s = g.standard_normal(BORDER_SAMPLE).astype(np.float32).astype(np.float64)
        q = np.quantile(s, np.linspace(0, 1, border_count + 1)[1:-1])
        out.append(np.unique(q.astype(np.float32).astype(np.float64)))
    return out


def make_borders(F: int, border_count: int, seed: int):
    """Uniform-quantile borders from a fixed-seed sample of the same distribution;
    NaN-bearing columns get the nan_mode=Min sentinel (border_count includes it)."""
    g = np.random.default_rng([seed, 1 << 31])
    h = F // 2
    S = np.empty((F, BORDER_SAMPLE), dtype=np.float32)
    S[:h] = g.standard_normal((h, BORDER_SAMPLE), dtype=np.float32)
    S[h:] = g.random((F - h, BORDER_SAMPLE), dtype=np.float32)
    out = []
    k = border_count - 1
    for f in range(F):
        q = np.quantile(S[f].astype(np.float64), np.linspace(0, 1, k + 2)[1:-1])
        b = np.unique(q.astype(np.float32).astype(np.float64))
        out.append(np.concatenate([[FMIN], b]))
    return out


def shard_bounds(n_total: int, world: int, rank: int):
    per = -(-n_total // world)
    per = -(-per // 8192) * 8192  # MVS-aligned shards
    lo = min(n_total, rank * per)
    hi = min(n_total, lo + per)
    return lo, hi - lo


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed region: NVML
    read-only queries every 10 ms (so even a short region gets samples), else
    nvidia-smi's 50 ms loop.  Rows: [index, sm MHz, max sm MHz, power W,
    active, hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap]."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        self.gpu = int(ids[gpu]) if gpu < len(ids) and ids[gpu].isdigit() else gpu
        self.rows = []
        self.proc = None
        self.stop = threading.Event()
        self.nvml = None

    def _sample_nvml(self, nv, h, mx):
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        try:
            pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
        except Exception:
            pw = float("nan")
        self.rows.append([str(self.gpu), str(sm), str(mx), f"{pw:.1f}", hex(rs)] +
                         ["Active" if rs & b else "Not Active" for b in bits])

    def _poll_nvml(self):
        while not self.stop.wait(0.01):
            try:
                self._sample_nvml(self.nvml, self.h, self.mx)
            except Exception as e:
                self.error = repr(e)

    def __enter__(self):
        self.error = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.nvml = nv
            self._sample_nvml(nv, self.h, self.mx)  # the region's first sample, taken synchronously
            self.t = threading.Thread(target=self._poll_nvml, daemon=True)
            self.t.start()
            return self
        except Exception as e:
            self.error = repr(e)
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.nvml:
            self.stop.set()
            self.t.join(timeout=2)
            try:
                self._sample_nvml(self.nvml, self.h, self.mx)  # and its last
                self.nvml.nvmlShutdown()
            except Exception as e:
                self.error = repr(e)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
            if self.error:
                out["error"] = self.error
            return out
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for k, nm in enumerate(names):
                if len(r) > 5 + k and r[5 + k].lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows),
                "source": "nvml" if self.nvml else "nvidia-smi"}


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the C restatement of the reference CPU path
# ---------------------------------------------------------------------------

def cpu_reference_run(args, X, y, trees: int, warm: int, budget_s: float):
    """The oracle (the C restatement of the reference CPU path, OpenMP over
    features as the reference's rayon loop) on the FULL workload: every row
    and feature, boosting trees at the config's depth, all host threads.
    `warm` untimed trees first; then `trees` timed trees, fewer when the
    warm-up tree's time says they would exceed `budget_s` (at least 3)."""
    from oracle import oracle as orc
    c5 = getattr(args, "config", 2) == 5
    borders = (make_borders5 if c5 else make_borders)(args.features, args.border_count, args.seed)
    bins = orc.quantize(X, borders)
    threads = os.cpu_count() or 1
    kw = dict(loss="RMSE" if c5 else "Logloss", depth=args.depth, learning_rate=0.05, l2_leaf_reg=3.0,
              score_function="Cosine", bootstrap_type="MVS" if c5 else "Bayesian", bagging_temperature=1.0,
              subsample=0.8, random_seed=0, boost_from_average=False, staged=False, n_threads=threads)
    counts = [len(b) for b in borders]
    if warm:
        t0 = time.perf_counter()
        orc.train(bins, counts, y, iterations=warm, **kw)
        per = (time.perf_counter() - t0) / warm
        trees = max(3, min(trees, int(budget_s / max(per, 1e-9))))
    t0 = time.perf_counter()
    orc.train(bins, counts, y, iterations=trees, **kw)
    dt = time.perf_counter() - t0
    return trees / dt, threads, dt, trees


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=10_000_000)
    ap.add_argument("--features", type=int, default=200)
    ap.add_argument("--depth", type=int, default=8)
    ap.add_argument("--border-count", type=int, default=128)
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--cpu-trees", type=int, default=3)
    ap.add_argument("--cpu-budget-s", type=float, default=60.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5],
                    help="BASELINE config: 2 (default) or 5 (RMSE 50M x 500, depth 10, MVS) on this file's "
                         "scalar session; 3 (MultiClass) or 4 (ranking) from bench_configs.py")
    ap.add_argument("--variant", default=None, help="config 3: onehot | bernoulli; config 4: yetirank | pairlogit | "
                                                         "yetirankpairwise | pairlogitpairwise")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config == 5:  # its shape unless overridden on the command line
        for k, v in (("rows", 50_000_000), ("features", 500), ("depth", 10)):
            if getattr(args, k) == ap.get_default(k):
                setattr(args, k, v)
    if args.config in (3, 4):
        import bench_configs
        if args.seed == 20261201:
            args.seed = 0
        (bench_configs.run_config3 if args.config == 3 else bench_configs.run_config4)(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    c5 = args.config == 5
    metric = "trees/sec at 50M x 500 depth-10 RMSE (MVS)" if c5 else "trees/sec at 10M x 200 depth-8 Logloss"
    loss, boot = ("RMSE", "MVS") if c5 else ("Logloss", "Bayesian")
    block = _block5 if c5 else _block
    base_cfg = {"workload": "config5: RMSE 50M x 500 N(0,1) f32, sparse linear target + noise, border_count 128, "
                            "depth 10, lr 0.05, MVS subsample 0.8, Cosine, l2 3" if c5 else
                            "config2: Logloss 10M x 200 f32 (half N(0,1), half U(0,1), 5% NaN), "
                            "border_count 128 (nan_mode Min), depth 8, lr 0.05, Bayesian T=1, Cosine, l2 3",
                "rows": args.rows, "features": args.features, "depth": args.depth,
                "border_count": args.border_count, "parallelism": f"doc-shard x{world}",
                "l2_flush": "inputs larger than L2 (%.1f GB of row-major bins re-read per tree)"
                            % (args.rows * -(-args.features // 32) * 32 / 1e9)}

    if args.impl == "reference":
        if rank != 0:
            return
        # the full workload (every row and feature); the timed trees are bounded
        # by a time budget so the run ends within a few minutes
        X, y = make_shard(0, args.rows, args.features, args.seed, block)
        tps, cores, dt, timed = cpu_reference_run(args, X, y, args.steps, 1, 2.0 * args.cpu_budget_s)
        sample = (f"C restatement of the reference CPU path (oracle/), full workload {args.rows} rows x "
                  f"{args.features} features at depth {args.depth}, {cores} threads: 1 warm-up tree, then "
                  f"{timed} boosting trees timed ({dt:.1f} s); no extrapolation")
        line = {"impl": "reference", "metric": metric, "value": tps, "unit": "trees/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1e3 / tps, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f64", "data": "synthetic", "config": base_cfg,
                "cpu_baseline": {"value": tps, "unit": "trees/s", "cores": cores, "kind": "port",
                                 "sample": sample, "timed_trees": timed},
                "e2e": {"value": tps, "unit": "trees/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import catboost_rs_b200 as cb

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    F = args.features
    row_offset, n = shard_bounds(args.rows, world, rank)
    X, y = make_shard(row_offset, n, F, args.seed, block)
    borders = (make_borders5 if c5 else make_borders)(F, args.border_count, args.seed)
    cols = [X[f] for f in range(F)]
    def fresh_uid():
        # an NCCL unique id serves one communicator: every session gets its own
        if world == 1:
            return None
        obj = [cb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    def open_session(sample_from_host: bool):
        uid = fresh_uid()
        rt = cb.B200Runtime()
        cfg = cb.DeviceTrainConfig(bootstrap_type=boot, bagging_temperature=1.0, sample_rate=0.8, rng_seed=0,
                                   bias=0.0, sample_from_host=sample_from_host, device=local_rank, rank=rank,
                                   world_size=world, row_offset=row_offset, n_total=args.rows,
                                   nccl_unique_id=uid)
        ok = rt.begin_device_training_raw(loss, args.depth, True, 1, "Cosine", cols, borders, None, n, F,
                                          max(len(b) for b in borders) + 1, LR_SEAM, 3.0, cfg)
        if not ok:
            raise RuntimeError(rt.decline_reason)
        return rt

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident throughput (value) -------------------------------
    rt = open_session(False)
    rt.set_profiling(True)  # per-kernel CUDA events; read after each tree's final sync
    for _ in range(args.warmup):
        rt.grow_tree_on_device(None, y, [], leaf_of_bytes=0, resident_approx=True)
    rt.timing_sum(reset=True)  # drop the warm-up trees
    barrier()
    with ClockSampler(local_rank) as clk:
        rt.mark(0)
        for _ in range(args.steps):
            rt.grow_tree_on_device(None, y, [], leaf_of_bytes=0, resident_approx=True)
        rt.mark(1)
        elapsed = rt.elapsed_ms(0, 1)
        barrier()
    # per-stage sums over the timed trees (each tree's event times are read
    # during the next tree's device work, so the loop above has no host reads)
    stage = rt.timing_sum()
    hist_ms, rows, launches = stage[1], stage[6], stage[7]
    elapsed = max_over_ranks(elapsed)
    rt.end_device_training()
    value = args.steps / (elapsed / 1e3)

    # histogram roofline: algorithmic bytes = rows x (F bins + 16 B g/h) + 4 B index per gathered row
    lvl0_rows = args.steps * n
    alg_bytes = rows * (F + 16) + (rows - lvl0_rows) * 4
    hist_launches = args.steps * args.depth
    achieved = alg_bytes / (hist_ms / 1e3) / 1e9 if hist_ms > 0 else None
    peak, peak_kind = peaks()
    dram_per_row, dram_cmd = hist_dram_bytes_per_row()
    if args.config != 2 or F != 200:  # the capture is of config 2's 200-feature rows
        dram_per_row = None

    # ---- end to end through the C ABI with host buffers (e2e) --------------
    e2e = None
    if not args.no_e2e:
        rt2 = open_session(True)
        pin = lambda shape, dt: torch.empty(shape, dtype=dt, pin_memory=True).numpy()  # noqa: E731
        # two pinned sample buffers, used in turn: the sample of tree t + 1 is
        # staged (cbgpu_stage_sample) before tree t grows, so its upload
        # overlaps tree t's device work
        rs = np.random.default_rng(7)
        samples = []
        for _ in range(2):
            smp = pin((n,), torch.float64)
            smp[:] = -np.log(rs.random(n))  # Bayesian-like multipliers; content does not change the cost
            samples.append(smp)
        lb = 1 if args.depth <= 8 else 2  # leaf id bytes the seam returns
        leaf_of = pin((n,), torch.uint8 if lb == 1 else torch.int16)
        import ctypes as C
        L = cb.load_library()
        D = args.depth
        sf = np.empty(D, np.int32)
        sb = np.empty(D, np.int32)
        ns = np.zeros(1, np.int32)
        lv = np.empty(1 << D, np.float64)
        yy = np.ascontiguousarray(y)

        def stage_sample(t):
            if L.cbgpu_stage_sample(rt2._s, samples[t & 1].ctypes.data, n):
                raise RuntimeError(cb._lib.last_error())

        def run(trees):
            # every tree's sample is uploaded inside the loop: the first before
            # tree 0, each later one while the tree before it grows
            stage_sample(0)
            for t in range(trees):
                if t + 1 < trees:
                    stage_sample(t + 1)
                rc = L.cbgpu_grow_tree(rt2._s, None, yy.ctypes.data, n, None, 0, sf.ctypes.data, sb.ctypes.data,
                                       ns.ctypes.data, lv.ctypes.data, leaf_of.ctypes.data, lb)
                if rc:
                    raise RuntimeError(cb._lib.last_error())
        run(args.warmup)
        barrier()
        rt2.mark(0)
        run(args.steps)
        rt2.mark(1)
        e_ms = max_over_ranks(rt2.elapsed_ms(0, 1))
        barrier()
        rt2.end_device_training()
        e2e = {"value": args.steps / (e_ms / 1e3), "unit": "trees/s", "h2d_bytes_per_step": int(n * 8),
               "d2h_bytes_per_step": int(lb * n + D * 8 + (1 << D) * 8),
               "path": "cbgpu_grow_tree with a pinned host bootstrap sample (sample_from_host, the cb-train "
                       "contract) uploaded and leaf ids (u8, u16 past depth 8) read back every tree; each "
                       "tree's sample is staged (cbgpu_stage_sample) while the tree before it grows, the "
                       "first one inside the timed region"}

    # ---- CPU baseline (rank 0, N=1 only) -------------------------------------
    cpu = None
    if world == 1 and not args.no_cpu:
        del cols
        tps, cores, dt, timed = cpu_reference_run(args, X, y, args.cpu_trees, 0, args.cpu_budget_s)
        cpu = {"value": tps, "unit": "trees/s", "cores": cores, "kind": "port",
               "sample": f"C restatement of the reference CPU path (oracle/) on the full workload "
                         f"({n} rows x {F} features, depth {args.depth}), {timed} boosting trees timed "
                         f"({dt:.1f} s, {cores} threads); no extrapolation"}

    if rank == 0:
        line = {"metric": metric, "value": value, "unit": "trees/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": elapsed / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int64",
                "data": "synthetic (seeded, config-%d shapes and distributions)" % args.config, "config": base_cfg,
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": (achieved / peak) if achieved else None,
                             "traffic": (dram_per_row * rows / hist_launches) if dram_per_row else None,
                             "traffic_unit": "bytes per launch",
                             "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of the eight "
                                                f"histogram launches of a 2M-row tree, {dram_per_row} B per "
                                                f"histogrammed row, scaled by rows per launch: {dram_cmd}")
                             if dram_per_row else "no capture of this workload's row width",
                             "limiter": "shared-memory reduction issue: 4 exact 32-bit red.shared per "
                                        "(row, feature); LSU pipe 70.6% of peak, top stall mio_throttle "
                                        "(ncu, 2M rows)",
                             "kernel": "hist_kernel", "peak_kind": peak_kind,
                             "algorithmic_bytes_per_launch": alg_bytes / hist_launches,
                             "avg_launch_ms": hist_ms / hist_launches},
                "stage_ms_per_tree": {k: float(stage[i] / args.steps) for i, k in
                                      enumerate(["tree", "hist", "derive_score", "partition", "der_bootstrap",
                                                 "collectives"])},
                "hist_rows_per_tree": rows / args.steps,
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
