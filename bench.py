#!/usr/bin/env python3
"""Benchmark: requests/s of the ensemble decode step on 1..8 B200 (one process per GPU).

Default workload = BASELINE config 5 ("scale-out"): 65,536 symbols hashed over
the GPUs (splitmix64 mod N), full 4-tower ensemble at the reduced dims D2
(hidden 256, proj 512, depth 4, 8 heads; the default dims hold 153 MB of state
per symbol and cannot hold 65,536 symbols), bf16 CastLinear weights, fp32 state,
Zipf(1.1) symbol arrivals, micro-batches of up to 4096 requests formed by the
reference's round rule, 79 N(0,1) float32 features per request. Weights are
seeded (hackathon_b200.weights, seed 0); data is synthetic.

A step = one micro-batch through the whole ensemble on each GPU. `value` is the
requests all ranks stepped in the K timed steps divided by the max-over-ranks
device time (CUDA events around K b2e_engine_submit_device calls and their join,
inputs already in HBM; consecutive steps overlap tower by tower). `e2e` is the
same metric through the C-ABI with HOST buffers (b2e_engine_submit / wait, two
steps in flight: H2D of slots and features, the step, D2H of predictions, all
inside the timed region). `latency_us.batch_*` is a step's submit-to-wait time
on that host path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload scaleout|d1-4096|d0-256]
    python bench.py --impl reference ...   # the reference's CPU path (oracle port), same metric
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

WORKLOADS = {
    # BASELINE config 5 at D2 (default)
    "scaleout": dict(preset="D2", symbols=65536, max_batch=4096, lp="bf16", zipf=1.1),
    # the north-star target row: 4096 symbols per step at D1
    "d1-4096": dict(preset="D1", symbols=4096, max_batch=4096, lp="bf16", zipf=None),
    # default dims, 256 symbols, one request each per step
    "d0-256": dict(preset="D0", symbols=256, max_batch=256, lp="bf16", zipf=None),
}
CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="scaleout")
    ap.add_argument("--symbols", type=int, default=None, help="override the symbol count")
    ap.add_argument("--linear-dtype", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--no-targets", action="store_true", help="skip the D1 / config 2-3 target runs")
    ap.add_argument("--quick", action="store_true",
                    help="device-timed steps only (no e2e, latency, roofline or CPU legs): for profiling")
    return ap.parse_args()


# ------------------------------------------------------------------ helpers


def step_bytes(cfg, lp: str, rows: int) -> int:
    """Algorithmic HBM bytes of one step: every weight once, plus per row its state
    read and written once, its features in and its 4 predictions out."""
    from hackathon_b200 import weights as W
    from hackathon_b200.engine import model_layout

    srow = sum(int(np.prod(shape)) * dt.itemsize for shape, dt in model_layout(cfg))
    return W.weight_bytes(cfg, lp) + rows * (2 * srow + cfg.num_features * 4 + 4 * 4 + 4)


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, device):
        import torch

        self.proc, self.path = None, None
        try:
            self.id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.id = str(device.index)

    def start(self, path: Path):
        self.path = path
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.id}", f"--query-gpu={CLOCK_QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce(x: float, op: str, world: int, device) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def make_batches(wl, n_symbols, world, rank, count, seed=0, backlog=None, info=None):
    """(slots per micro-batch on this rank, capacity) for `count` micro-batches.
    `backlog`: Zipf arrivals generated (default max(10M, 4M per GPU)).

    Per-GPU work stays fixed as the GPU count grows (weak scaling): only the
    stream's full micro-batches (max_batch distinct symbols) are used, in stream
    order, and repeated in that order when the run needs more than the stream
    yields. Under Zipf arrivals a rank that owns few symbols runs out of pending
    symbols after a while (at 8 GPUs, 8,192 symbols per rank: ~128 full
    micro-batches from 32M arrivals); `info["distinct"]` = the full ones used."""
    from hackathon_b200 import batcher as B

    mine, slot_of = B.shard_slots(n_symbols, world, rank)
    if wl["zipf"] is None:
        # every owned symbol once per step, max_batch per micro-batch
        per = np.arange(len(mine), dtype=np.int32)
        out = []
        rng = np.random.default_rng(seed + rank)
        while len(out) < count:
            perm = rng.permutation(per)
            for c in range(0, len(perm), wl["max_batch"]):
                out.append(perm[c:c + wl["max_batch"]])
        return out[:count], len(mine)
    # A deep backlog keeps >= max_batch symbols pending, so every micro-batch is
    # full: 10M arrivals (BASELINE config 5's stream), at least 4M per GPU.
    need = backlog or max(10_000_000, 4_000_000 * world)
    stream = B.zipf_stream(n_symbols, need, wl["zipf"], seed)
    own = stream[B.owner(stream, world) == rank]
    out = [slot_of[own[idx]].astype(np.int32)
           for idx in B.continuous_batches(own, wl["max_batch"], limit=count)]
    full = [b for b in out if len(b) == wl["max_batch"]]
    if full and len(full) < len(out):
        out = [full[i % len(full)] for i in range(count)]
    if info is not None:
        info["distinct"] = len(full) if full else len(out)
    return out, len(mine)


def read_traffic_per_row(name: str):
    """dram bytes per row of the dominant kernel from the committed ncu summary
    profiles/<name>.txt (its `traffic_bytes_per_row:` line)."""
    p = REPO / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_row:"):
            return float(line.split(":", 1)[1])
    return None


# ------------------------------------------------------------- reference arm


def metric_name(wl) -> str:
    return "requests/s (full 4-tower ensemble decode step, micro-batches <= %d)" % wl["max_batch"]


# ---- the CPU port on every host core: rows are independent (no operator mixes
# rows, example_model.py:422-427), so each worker process steps its own share of
# the sample's rows with its own oracle and state. Workers start with spawn.

_W = {}


def _port_init(preset, rows, seed):
    try:  # one BLAS thread per worker process: the processes are the parallelism
        from threadpoolctl import threadpool_limits

        _W["limits"] = threadpool_limits(1)
    except ImportError:
        pass
    from hackathon_b200 import config as C
    from hackathon_b200 import weights as Wt
    from oracle import model as O

    cfg = C.PRESETS[preset]
    _W["orc"] = O.Oracle(cfg, Wt.generate_model(cfg, seed=seed))
    _W["state"] = O.init_state(cfg, rows)


def _port_step(feats):
    p, _W["state"] = _W["orc"].step(feats, _W["state"])
    return p


class PortPool:
    """The numpy oracle (the reference's arithmetic in fp32) stepping `rows` rows
    split over `workers` processes; step(feats) returns the predictions."""

    def __init__(self, preset, rows, workers=None):
        import multiprocessing as mp
        from concurrent.futures import ProcessPoolExecutor

        self.workers = max(1, min(workers or os.cpu_count() or 1, rows))
        self.bounds = np.linspace(0, rows, self.workers + 1).astype(int)
        self.pools = [ProcessPoolExecutor(1, mp_context=mp.get_context("spawn"), initializer=_port_init,
                                          initargs=(preset, int(b - a), 0))
                      for a, b in zip(self.bounds[:-1], self.bounds[1:])]

    def step(self, feats):
        futs = [p.submit(_port_step, feats[a:b]) for p, a, b in zip(self.pools, self.bounds[:-1], self.bounds[1:])]
        return np.concatenate([f.result() for f in futs])

    def close(self):
        for p in self.pools:
            p.shutdown()


def run_reference(a, wl):
    """The reference's CPU path (the oracle port: numpy float32, all host threads)
    on a bounded sample of the same workload; rank 0 only."""
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return
    from hackathon_b200 import config as C

    cfg = C.PRESETS[wl["preset"]]
    sample_rows = 256 if wl["preset"] != "D0" else 4
    pool = PortPool(wl["preset"], sample_rows)
    rng = np.random.default_rng(0)
    times = []
    for i in range(a.warmup + a.steps):
        feats = rng.standard_normal((sample_rows, cfg.num_features), dtype=np.float32)
        t0 = time.perf_counter()
        pool.step(feats)
        if i >= a.warmup:
            times.append(time.perf_counter() - t0)
    pool.close()
    total = sum(times)
    value = sample_rows * len(times) / total
    cores = pool.workers
    cpu = {"value": value, "unit": "requests/s", "cores": cores, "kind": "port",
           "sample": f"{len(times)} steps of {sample_rows} symbols at {wl['preset']} (fp32 oracle, numpy, rows split "
                     f"over {cores} processes)"}
    line = {"impl": "reference", "metric": metric_name(wl), "value": value,
            "unit": "requests/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": 1e3 * total / len(times), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": a.workload, "dims": wl["preset"], "symbols": wl["symbols"],
                       "max_batch": wl["max_batch"], "rows_per_step": sample_rows,
                       "note": "a bounded sample: each step is one micro-batch of rows_per_step symbols"},
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "requests/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ main arm


def main():
    a = parse()
    wl = dict(WORKLOADS[a.workload])
    if a.linear_dtype:
        wl["lp"] = a.linear_dtype
    if a.symbols:
        wl["symbols"] = a.symbols
    if a.impl == "reference":
        run_reference(a, wl)
        return
    import torch

    from hackathon_b200 import config as C
    from hackathon_b200 import weights as Wt
    from hackathon_b200.engine import EnsembleEngine

    world, rank, local = dist_setup(a.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = C.PRESETS[wl["preset"]]
    n_sym = wl["symbols"]
    K, Wm = a.steps, max(3, a.warmup)
    binfo = {}
    batches, capacity = make_batches(wl, n_sym, world, rank, Wm + 2 * K + 2, info=binfo)
    sd = Wt.generate_model(cfg, seed=0)
    eng = EnsembleEngine(cfg, sd, device=local, linear_dtype=wl["lp"], capacity=capacity,
                         max_batch=wl["max_batch"], graphs=not a.no_graphs)
    del sd
    rng = np.random.default_rng(1000 + rank)
    F = cfg.num_features
    feats = [rng.standard_normal((len(b), F), dtype=np.float32) for b in batches]
    d_slots = [torch.from_numpy(b).to(dev) for b in batches]
    d_feats = [torch.from_numpy(f).to(dev) for f in feats]
    preds = [torch.empty(wl["max_batch"], 4, device=dev) for _ in range(max(K, Wm))]
    stream = torch.cuda.current_stream(dev)

    # ---- device-resident timing (value): b2e_engine_submit_device per micro-batch
    # (consecutive steps overlap tower by tower), one join at the end
    for i in range(Wm):
        eng.submit_device(d_slots[i], d_feats[i], preds[i], len(batches[i]), stream=stream)
    eng.join_device(stream=stream)
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(dev)
    clock_dir = tempfile.mkdtemp(prefix="b2e_clocks_")
    clocks.start(Path(clock_dir) / f"clocks_rank{rank}.csv")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    barrier(world)
    ev[0].record(stream)
    rows = 0
    for k in range(K):
        i = Wm + k
        eng.submit_device(d_slots[i], d_feats[i], preds[k], len(batches[i]), stream=stream)
        rows += len(batches[i])
    eng.join_device(stream=stream)
    ev[1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    t_ms = ev[0].elapsed_time(ev[1])
    assert eng.device_error() == 0
    t_max = allreduce(t_ms, "max", world, dev)
    rows_all = allreduce(float(rows), "sum", world, dev)
    value = rows_all / (t_max / 1e3)
    distinct = -allreduce(-float(binfo.get("distinct", len(batches))), "max", world, dev)  # min over ranks

    if a.quick:
        if rank == 0:
            print(json.dumps({"quick": True, "value": value, "unit": "requests/s", "ms_per_step": t_max / K,
                              "launches_per_step": eng.launches_per_step(wl["max_batch"]) + 1}), flush=True)
        eng.close()
        return

    # ---- end to end through the C-ABI with host buffers (e2e): b2e_engine_submit
    # / b2e_engine_wait with two steps in flight, so a step's host->device copy
    # and towers overlap the previous step's; each step's latency is the time
    # from its submit to the return of its wait
    barrier(world)
    t0 = time.perf_counter()
    h2d = d2h = 0
    t_sub, t_done = [], []
    for k in range(K):
        i = Wm + K + k
        t_sub.append(time.perf_counter())
        eng.submit(batches[i], feats[i])
        if k:
            eng.wait()
            t_done.append(time.perf_counter())
        h2d += 4 + 4 * len(batches[i]) + 4 * F * len(batches[i])
        d2h += 16 * len(batches[i])
    eng.wait()
    t_done.append(time.perf_counter())
    e2e_s = time.perf_counter() - t0
    step_ms = [(d - u) * 1e3 for u, d in zip(t_sub, t_done)]
    e2e_rows = float(sum(len(batches[Wm + K + k]) for k in range(K)))
    e2e_max = allreduce(e2e_s, "max", world, dev)
    e2e_val = allreduce(e2e_rows, "sum", world, dev) / e2e_max

    # ---- single-request latency through the C-ABI (host buffers, synchronous)
    lat = []
    one = np.zeros((1, F), np.float32)
    for i in range(220):
        t1 = time.perf_counter()
        eng.step(batches[0][i % len(batches[0]):i % len(batches[0]) + 1], one)
        lat.append((time.perf_counter() - t1) * 1e6)
    lat = np.asarray(lat[20:])

    # ---- roofline of the dominant state kernel, timed alone on its stream
    roof = None
    if rank == 0:
        roof = dominant_kernel_roofline(cfg, wl, dev, K)
    launches = eng.launches_per_step(wl["max_batch"])
    nb = step_bytes(cfg, wl["lp"], int(np.mean([len(batches[Wm + k]) for k in range(K)])))
    lat_rows, lat_cl = eng.latency_rows()

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(cfg, wl)
    ingest = ingest_rate(F) if rank == 0 and world == 1 and not a.no_targets else None

    per_req = np.repeat(step_ms, [len(batches[Wm + K + k]) for k in range(len(step_ms))])
    tg = None
    if rank == 0 and world == 1 and not a.no_targets:
        eng.close()  # the scale-out state table (119 GB) makes room for the target runs
        peak = roof["peak"] if roof else 6650.0
        tg = targets(dev, peak, K)
    if rank == 0:
        line = {
            "metric": metric_name(wl),
            "value": value, "unit": "requests/s", "n_gpus": world, "steps": K, "warmup": Wm,
            "ms_per_step": t_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 state, %s weights" % wl["lp"], "data": "synthetic (seeded weights, N(0,1) features)",
            "config": {"workload": a.workload, "dims": wl["preset"], "hidden": cfg.hidden_size,
                       "proj": cfg.proj_size, "depth": cfg.tower_depth, "heads": cfg.num_heads,
                       "symbols": n_sym, "symbols_per_gpu": capacity, "max_batch": wl["max_batch"],
                       "arrivals": f"Zipf({wl['zipf']})" if wl["zipf"] else "uniform, every symbol once per round",
                       "micro_batches": f"full ({wl['max_batch']} distinct symbols); the stream's first {int(distinct)} "
                                        f"per rank (fewest over ranks), reused in order when a run needs more",
                       "parallelism": f"symbol-sharded x{world} (splitmix64 mod N), no collective",
                       "l2": "inputs larger than L2: %.1f GB of state streamed per step" % (nb / 1e9)},
            "latency_us": {"batch_p50": float(np.percentile(per_req, 50) * 1e3),
                           "batch_p99": float(np.percentile(per_req, 99) * 1e3),
                           "single_request_p50": float(np.percentile(lat, 50)),
                           "single_request_p99": float(np.percentile(lat, 99)),
                           "single_request_path": (f"one kernel, {lat_cl}-CTA cluster per tower" if lat_rows
                                                   else "batch graph")},
            "hbm_gbs_step": nb / (t_max / K / 1e3) / 1e9,
            "e2e": {"value": e2e_val, "unit": "requests/s", "h2d_bytes_per_step": h2d // K,
                    "d2h_bytes_per_step": d2h // K},
            "gpu_launches": (launches + 1) * K,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clk,
            "targets": tg,
            "ingest": ingest,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def dominant_kernel_roofline(cfg, wl, dev, K):
    """Mamba2's state step - the largest state stream of the step, the bulk-copy
    streaming kernel the engine runs (ssm_cols dispatches to it) - timed alone
    with CUDA events on its stream at one engine launch's shape."""
    import torch

    from hackathon_b200 import kernels as KR

    peaks = {}
    pk = REPO / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = float(peaks.get("hbm_gbs", 6650.0))
    rows = wl["max_batch"]
    nh, hs, bc = cfg.mamba_heads, cfg.mamba_head_size, cfg.mamba_bc_size
    g = torch.Generator(device=dev).manual_seed(0)
    ssm = torch.randn(rows, nh, hs, bc, device=dev, generator=g)
    x = torch.randn(rows, nh, hs, device=dev, generator=g)
    b = torch.randn(rows, bc, device=dev, generator=g)
    c = torch.randn(rows, bc, device=dev, generator=g)
    dt = torch.rand(rows, nh, device=dev, generator=g)
    dc = torch.rand(rows, nh, device=dev, generator=g)
    s = torch.cuda.current_stream(dev)
    per_row = 2 * nh * hs * bc * 4 + (nh * hs * 2 + 2 * bc + 2 * nh) * 4

    def launch_s(waves):
        # waves 0: the persistent grid the ensemble step launches; 8: the
        # short-CTA grid of a state step streaming alone (the default there)
        prev = KR.set_state_kernel_waves(waves)
        try:
            for _ in range(3):
                KR.mamba2_step(ssm, x, b, c, dt, dc, None)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = max(10, K)
            torch.cuda.synchronize()
            e0.record(s)
            for _ in range(n):
                KR.mamba2_step(ssm, x, b, c, dt, dc, None)
            e1.record(s)
            torch.cuda.synchronize()
        finally:
            KR.set_state_kernel_waves(prev)
        return e0.elapsed_time(e1) / n / 1e3

    t = launch_s(0)
    t_alone = launch_s(8)
    achieved = rows * per_row / t / 1e9
    alone = rows * per_row / t_alone / 1e9
    tr = read_traffic_per_row("ssm_bulk_d2")
    return {"kernel": "ssm_bulk_kernel (Mamba2 state step, bulk-copy streaming), the step's persistent grid",
            "bound": "hbm", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak, "traffic": None if tr is None else tr * rows,
            "bytes_per_launch": rows * per_row, "launch_us": t * 1e6,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if pk.exists() else "fallback 6650 GB/s",
            "standalone": {"grid": "short CTAs, ~8 waves of two per SM (b2e_mamba2_step's default)",
                           "achieved": alone, "frac": alone / peak, "launch_us": t_alone * 1e6}}


def _lat(eng, slots, F, n=220, skip=20):
    """Single-request latency through the host API (b2e_engine_step), microseconds:
    (p50, p99) over n - skip calls, rows at the given slots in turn."""
    one = np.zeros((1, F), np.float32)
    lat = []
    for i in range(n):
        s = slots[i % len(slots)]
        t1 = time.perf_counter()
        eng.step(np.asarray([s], np.int32), one)
        lat.append((time.perf_counter() - t1) * 1e6)
    lat = np.asarray(lat[skip:])
    return float(np.percentile(lat, 50)), float(np.percentile(lat, 99))


def _device_steps(step, K, W, stream):
    """Mean ms of one step over K device-timed steps after W warm-up ones."""
    import torch

    for _ in range(W):
        step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(K):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / K


def ingest_rate(F, n_requests=32768, per_line=16, n_symbols=256):
    """Host side of the request path, per request (microseconds): the native
    ingest (hackathon_b200.ingest.RequestIngest: protocol JSON lines straight into
    per-symbol queues, then micro-batches of up to 4096 rows as float32 arrays)
    beside the reference's way - json.loads per line, a Python list of floats per
    request into per-symbol queues, np.asarray per request (protocol.py:86-103,
    client.py:156-173, example_model.py:854-855) - on the same bytes; and
    response encoding (b2e_encode_response against json.dumps of the response)."""
    from hackathon_b200.ingest import RequestIngest, encode_response

    rng = np.random.default_rng(7)
    lines = []
    uid = 0
    for i in range(n_requests // per_line):
        syms = [f"SYM_{(i * per_line + j) % n_symbols:03d}" for j in range(per_line)]
        feats = rng.standard_normal((per_line, F)).astype(np.float32).tolist()
        d = {"unique_ids": list(range(uid, uid + per_line)), "symbols": syms, "features": feats,
             "timestamp": 1.5, "message_type": "inference_request"}
        uid += per_line
        lines.append((json.dumps(d) + "\n").encode())
    data = b"".join(lines)
    out = {"requests": n_requests, "requests_per_line": per_line, "bytes": len(data)}
    # 64 KB reads (a socket's) on one thread and on the host's threads; 1 MB reads (a backlog)
    for name, chunk, threads in (("native_us_per_request_64k_reads_1thread", 1 << 16, 1),
                                 ("native_us_per_request_64k_reads", 1 << 16, None),
                                 ("native_us_per_request_1m_reads", 1 << 20, None)):
        ing = RequestIngest(F, max_queue_size=0, threads=threads)
        t0 = time.perf_counter()
        for i in range(0, len(data), chunk):
            ing.feed(data[i:i + chunk])
        got = 0
        while True:
            rows = ing.take_batch(4096)
            if len(rows.unique_ids) == 0:
                break
            got += len(rows.unique_ids)
        dt = time.perf_counter() - t0
        ing.close()
        assert got == n_requests, (got, n_requests)
        out[name] = dt / n_requests * 1e6
    t0 = time.perf_counter()
    queues = {}
    for ln in lines:
        d = json.loads(ln.decode("utf-8").strip())
        for u, sym, f in zip(d["unique_ids"], d["symbols"], d["features"]):
            queues.setdefault(sym, []).append((u, f))
    rows = [np.asarray(f, np.float32) for q in queues.values() for _, f in q]
    out["python_json_us_per_request"] = (time.perf_counter() - t0) / n_requests * 1e6
    assert len(rows) == n_requests
    preds = rng.standard_normal((4096, 4)).astype(np.float32)
    ids = np.arange(4096, dtype=np.int64)
    t0 = time.perf_counter()
    for _ in range(8):
        encode_response(ids, preds, 1.5)
    out["native_encode_us_per_answer"] = (time.perf_counter() - t0) / (8 * 4096) * 1e6
    t0 = time.perf_counter()
    for _ in range(8):
        json.dumps({"unique_ids": ids.tolist(), "predictions": preds.tolist(), "client_timestamp": 1.5,
                    "message_type": "inference_response"})
    out["python_json_encode_us_per_answer"] = (time.perf_counter() - t0) / (8 * 4096) * 1e6
    out["host_threads"] = os.cpu_count()
    return out


def client_rate(dev, n_symbols=4096, calls=20):
    """The drop-in API itself: B200InferenceClient.process_batch (example_model.py:769-905)
    at D2 dims with bf16 weights, every call one request for each of n_symbols
    symbols (PendingRequest objects with Python lists of 79 floats, as the
    reference client queues them): wall-clock requests/s and ms per call, host
    work (grouping, np.asarray of the feature lists, the answer lists) included."""
    from hackathon_b200 import config as C
    from hackathon_b200 import weights as Wt
    from hackathon_b200.client import B200InferenceClient, PendingRequest

    cfg = C.D2
    cl = B200InferenceClient(n_symbols, config=cfg, weights=Wt.generate_model(cfg, seed=0), linear_dtype="bf16",
                             devices=[dev.index])
    rng = np.random.default_rng(11)
    uid = 0
    batches = []
    for _ in range(calls + 3):
        f = rng.standard_normal((n_symbols, cfg.num_features)).astype(np.float32).tolist()
        batches.append({f"SYM_{i:05d}": [PendingRequest(uid + i, f"SYM_{i:05d}", f[i], 0.0)] for i in range(n_symbols)})
        uid += n_symbols
    for b in batches[:3]:
        cl.process_batch(b)
    t0 = time.perf_counter()
    for b in batches[3:]:
        resp = cl.process_batch(b)
    dt = time.perf_counter() - t0
    assert len(resp.unique_ids) == n_symbols
    for e in cl.engines:
        e.close()
    return {"requests_per_s": calls * n_symbols / dt, "ms_per_call": dt / calls * 1e3, "symbols_per_call": n_symbols,
            "dims": "D2", "weights": "bf16"}


def _device_submits(eng, slots, feats, rows, K, W, stream):
    """Mean ms of one step over K device-timed b2e_engine_submit_device steps and
    their join, after W warm-up ones."""
    import torch

    preds = [torch.empty(rows, 4, device=slots.device) for _ in range(max(K, W))]
    for i in range(W):
        eng.submit_device(slots, feats, preds[i], rows, stream=stream)
    eng.join_device(stream=stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(K):
        eng.submit_device(slots, feats, preds[i], rows, stream=stream)
    eng.join_device(stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / K


def targets(dev, peak, K):
    """The north_star's target row and BASELINE configs 2 and 3, beside the headline:
    * d1_4096: the full ensemble at D1 (depth 12), 4096 symbols per step, bf16
      weights, fp32 state: requests/s and the whole step's HBM fraction;
    * single-request latency (host API, one row) at D1 and D2, and at the default
      dims (config 1's shape);
    * process_batch: the drop-in client API's requests/s with 4096 symbols a call;
    * config2 / config3: the Mamba2 layer (d_state 64, stated a / dt fills), the
      RetNet layer (4 heads of 64, gamma_h = 1 - 2^(-5-h)) and the xLSTM layer
      whose mLSTM cell has 4 heads of 64, each 4096 symbols x 1,000 steps, bf16
      weights: ms per step and HBM fraction of weights + state read and written."""
    import torch

    from hackathon_b200 import config as C
    from hackathon_b200 import weights as Wt
    from hackathon_b200.engine import EnsembleEngine, LayerEngine, leaf_layout

    out = {}
    stream = torch.cuda.current_stream(dev)
    cfg = C.D1
    sd = Wt.generate_model(cfg, seed=0)
    rows = 4096
    eng = EnsembleEngine(cfg, sd, device=dev.index, linear_dtype="bf16", capacity=rows, max_batch=rows)
    rng = np.random.default_rng(3)
    slots = torch.from_numpy(rng.permutation(rows).astype(np.int32)).to(dev)
    feats = torch.from_numpy(rng.standard_normal((rows, cfg.num_features), dtype=np.float32)).to(dev)
    ms = _device_submits(eng, slots, feats, rows, max(K, 10), 3, stream)
    assert eng.device_error() == 0
    nb = step_bytes(cfg, "bf16", rows)
    out["d1_4096"] = {"requests_per_s": rows / (ms / 1e3), "ms_per_step": ms, "bytes_per_step": nb,
                      "hbm_gbs": nb / (ms / 1e3) / 1e9, "hbm_frac": nb / (ms / 1e3) / 1e9 / peak,
                      "launches_per_step": eng.launches_per_step(rows)}
    lr, cl = eng.latency_rows()
    p50, p99 = _lat(eng, list(range(64)), cfg.num_features)
    out["d1_single_request_us"] = {"p50": p50, "p99": p99, "path": f"one kernel, {cl}-CTA cluster per tower"
                                   if lr else "batch graph"}
    eng.close()
    del sd
    # BASELINE config 1's shape: one request at a time at the default dims (batch
    # graph: the latency kernel's stage slices do not fit at hidden 2048)
    cfg0 = C.D0
    sd = Wt.generate_model(cfg0, seed=0)
    eng = EnsembleEngine(cfg0, sd, device=dev.index, linear_dtype="bf16", capacity=16, max_batch=16)
    del sd
    lr, cl = eng.latency_rows()
    p50, p99 = _lat(eng, list(range(16)), cfg0.num_features)
    out["config1_single_request_us"] = {"p50": p50, "p99": p99, "dims": "D0 (hidden 2048, depth 12)",
                                        "weights": "bf16", "path": f"one kernel, {cl}-CTA cluster per tower"
                                        if lr else "batch graph"}
    eng.close()
    out["process_batch"] = client_rate(dev)
    for name, kinds in (("config2", ["mamba2"]), ("config3", ["retnet", "xlstm"])):
        res = {}
        for kind in kinds:
            mc, msd = Wt.micro_layer(kind, seed=0)
            le = LayerEngine(kind, mc, msd, device=dev.index, linear_dtype="bf16", capacity=rows, max_batch=rows)
            x = torch.from_numpy(rng.standard_normal((rows, mc.hidden_size), dtype=np.float32)).to(dev)
            y = torch.empty(rows, mc.hidden_size, device=dev)
            ms = _device_steps(lambda: le.step_device(slots, x, y), 1000, 5, stream)
            srow = sum(int(np.prod(sh)) * dt.itemsize for sh, dt in leaf_layout(kind, mc))
            nbk = Wt.layer_weight_bytes(kind, mc, "bf16") + rows * (2 * srow + 2 * mc.hidden_size * 4)
            res[kind] = {"ms_per_step": ms, "steps": 1000, "symbols": rows, "bytes_per_step": nbk,
                         "hbm_frac": nbk / (ms / 1e3) / 1e9 / peak}
            le.close()
        out[name] = res
    return out


def cpu_baseline(cfg, wl):
    """The reference's CPU arithmetic (the numpy oracle port, fp32) on a bounded
    sample of this workload: 256-symbol micro-batches, the rows split over every
    host core (spawned processes), for ~10 s."""
    preset = wl["preset"]
    rows = 256 if cfg.hidden_size <= 512 else 2
    pool = PortPool(preset, rows)
    rng = np.random.default_rng(0)
    pool.step(rng.standard_normal((rows, cfg.num_features), dtype=np.float32))
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0:
        pool.step(rng.standard_normal((rows, cfg.num_features), dtype=np.float32))
        n += 1
    dt = time.perf_counter() - t0
    pool.close()
    return {"value": rows * n / dt, "unit": "requests/s", "cores": pool.workers, "kind": "port",
            "sample": f"{n} micro-batches of {rows} symbols, fp32 numpy oracle, rows split over {pool.workers} "
                      f"processes, {dt:.1f} s"}


if __name__ == "__main__":
    main()
