"""Profiling helpers: single-kernel cases for ncu, and summaries of its output.

    python -m hackathon_b200.profiling cell --kind mamba2 --rows 4096 --heads 8 --sh 64 --sk 128
        run one state-step kernel `--reps` times on a dense state (for ncu -k)
    python -m hackathon_b200.profiling layer --kind xlstm --rows 4096 --reps 4 [--micro]
        one layer at the bench's dims `--reps` steps (its kernels, for ncu -k);
        --micro: BASELINE config 2 / 3's layer
    python -m hackathon_b200.profiling step --preset D2 --rows 2048 --reps 4
        the whole ensemble step on device buffers (its GEMMs, for ncu -k)
    python -m hackathon_b200.profiling latency --preset D2 --reps 8
        single-request steps on the one-kernel latency path (for ncu -k)
    python -m hackathon_b200.profiling latency-trace --preset D2
        the same steps through the trace build (lib/libb2e_trace.so): per tower
        and stage kind, the wait at the cluster barrier, the compute warps' work,
        the producer warp's copies of the next stage (beside that work), and the
        cluster arrive
    python -m hackathon_b200.profiling launches <launch list csv>
        per-kernel launches, total time and share of an ncu launch list
    python -m hackathon_b200.profiling metrics <raw csv from ncu -i ... --page raw --csv>
        the DRAM/tensor/occupancy counters used in the roofline, per kernel
"""

from __future__ import annotations

import argparse
import collections
import csv
import sys

SCALE = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3}
METRICS = ("gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum",
           "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "dram__throughput.avg.pct_of_peak_sustained_elapsed",
           "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active", "sm__warps_active.avg.pct_of_peak_sustained_active",
           "launch__registers_per_thread", "launch__grid_size", "launch__block_size",
           "sm__throughput.avg.pct_of_peak_sustained_elapsed")


def _short(name: str) -> str:
    return name.split("(")[0].replace("(anonymous namespace)::", "").replace("void ", "")


def launches(path: str) -> None:
    rows = list(csv.reader(open(path)))
    hdr, agg = None, collections.defaultdict(lambda: [0, 0.0])
    for r in rows:
        if r and r[0] == "ID":
            hdr = r
            continue
        if not hdr or len(r) != len(hdr):
            continue
        d = dict(zip(hdr, r))
        if d["Metric Name"] != "gpu__time_duration.sum":
            continue
        us = float(d["Metric Value"].replace(",", "")) * SCALE.get(d["Metric Unit"], 1e-3)
        agg[_short(d["Kernel Name"])][0] += 1
        agg[_short(d["Kernel Name"])][1] += us
    total = sum(v[1] for v in agg.values())
    print(f"{'kernel':52s} {'launches':>8s} {'total us':>10s} {'share':>6s}")
    for k, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        print(f"{k:52s} {n:8d} {t:10.1f} {100 * t / total:5.1f}%")
    print(f"{'total':52s} {sum(v[0] for v in agg.values()):8d} {total:10.1f}")


def metrics(path: str) -> None:
    rows = list(csv.reader(open(path)))
    hdr = rows[0]
    units = rows[1] if len(rows) > 1 else []
    for r in rows[2:]:
        d = dict(zip(hdr, r))
        print(_short(d.get("Kernel Name", "?")))
        for m in METRICS:
            if m in d:
                u = units[hdr.index(m)] if units else ""
                print(f"  {m} = {d[m]} {u}")


def cell(kind: str, rows: int, heads: int, sh: int, sk: int, reps: int, waves: int | None = None) -> None:
    """`reps` launches of one fused state step on a dense state; `waves` picks the
    state kernel's grid (0: the ensemble step's persistent grid; None: the
    library's default for a step launched alone)."""
    import torch

    from . import kernels as K

    if waves is not None:
        K.set_state_kernel_waves(waves)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    state = torch.randn(rows, heads, sh, sk, device=dev, generator=g)
    if kind == "mamba2":
        args = (torch.randn(rows, heads, sh, device=dev, generator=g), torch.randn(rows, sk, device=dev, generator=g),
                torch.randn(rows, sk, device=dev, generator=g), torch.rand(rows, heads, device=dev, generator=g),
                torch.rand(rows, heads, device=dev, generator=g))
        fn = K.mamba2_step
    elif kind == "mlstm":
        args = (torch.randn(rows, heads, sh, device=dev, generator=g), torch.randn(rows, heads, sh, device=dev, generator=g),
                torch.randn(rows, heads, sk, device=dev, generator=g), torch.rand(rows, heads, device=dev, generator=g),
                torch.rand(rows, heads, device=dev, generator=g))
        fn = K.mlstm_step
    elif kind == "retnet":
        args = (torch.randn(rows, heads, sh, device=dev, generator=g), torch.randn(rows, heads, sk, device=dev, generator=g),
                torch.randn(rows, heads, sh, device=dev, generator=g), torch.rand(heads, device=dev, generator=g))
        fn = K.retnet_step
    else:
        raise SystemExit(f"unknown kind {kind}")
    for _ in range(reps):
        fn(state, *args, None)
    torch.cuda.synchronize()
    print(f"{kind} rows={rows} heads={heads} sh={sh} sk={sk} waves={waves}: {reps} launches, "
          f"state {state.numel() * 4 / 1e9:.2f} GB")


def layer(kind: str, rows: int, reps: int, dtype: str, micro: bool = False) -> None:
    """One layer (xlstm / mamba2 / retnet / hawk) at the bench's dims (D2), `reps`
    steps over `rows` rows with random slots: its kernels at their bench shapes,
    with only that layer's state on the device. micro: the layer of BASELINE
    config 2 (mamba2) or 3 (retnet, xlstm) with its stated fills instead."""
    import numpy as np
    import torch

    from . import config as C
    from . import weights as W
    from .engine import LayerEngine

    if micro:
        cfg, sd = W.micro_layer(kind, seed=0)
    else:
        cfg = C.D2
        sd = W.generate(W.layer_specs(kind, "", cfg), seed=0)
    dev = torch.device("cuda", 0)
    eng = LayerEngine(kind, cfg, sd, linear_dtype=dtype, capacity=rows, max_batch=rows)
    slots = torch.from_numpy(np.random.default_rng(0).permutation(rows).astype(np.int32)).to(dev)
    x = torch.randn(rows, cfg.hidden_size, device=dev)
    y = torch.empty_like(x)
    for _ in range(reps):
        eng.step_device(slots, x, y)
    torch.cuda.synchronize()
    dims = "its config's dims" if micro else "D2"
    print(f"{kind} layer at {dims}, rows={rows}: {reps} steps, state {eng.slot_bytes * rows / 1e9:.2f} GB")
    eng.close()


def linear(m: int, k: int, n: int, reps: int, dtype: str) -> None:
    import torch

    from . import kernels as K

    dev = torch.device("cuda", 0)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[dtype]
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(m, k, device=dev, generator=g).to(dt)
    w = (torch.randn(n, k, device=dev, generator=g) * k ** -0.5).to(dt)
    b = torch.zeros(n, device=dev, dtype=dt)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(reps):
        K.cast_linear(x, w, b, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    print(f"linear {dtype} m={m} k={k} n={n}: {reps} launches")


def step(preset: str, rows: int, reps: int, dtype: str) -> None:
    """The whole ensemble step on device buffers, `reps` times (its GEMMs and
    state kernels, for ncu -k)."""
    import numpy as np
    import torch

    from . import config as C
    from . import weights as W
    from .engine import EnsembleEngine

    cfg = C.PRESETS[preset]
    eng = EnsembleEngine(cfg, W.generate_model(cfg, 0), linear_dtype=dtype, capacity=rows, max_batch=rows)
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    slots = torch.from_numpy(rng.permutation(rows).astype(np.int32)).to(dev)
    feats = torch.from_numpy(rng.standard_normal((rows, cfg.num_features), dtype=np.float32)).to(dev)
    preds = torch.empty(rows, 4, device=dev)
    for _ in range(reps):
        eng.step_device(slots, feats, preds, rows)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    print(f"step {preset} {dtype} rows={rows}: {reps} steps, {eng.launches_per_step(rows)} kernels each")
    eng.close()


def latency(preset: str, reps: int, dtype: str) -> None:
    """`reps` single-request host steps (the one-kernel latency path, for ncu -k)."""
    import numpy as np

    from . import config as C
    from . import weights as W
    from .engine import EnsembleEngine

    cfg = C.PRESETS[preset]
    eng = EnsembleEngine(cfg, W.generate_model(cfg, 0), linear_dtype=dtype, capacity=16, max_batch=16)
    one = np.zeros((1, cfg.num_features), np.float32)
    for i in range(reps):
        eng.step(np.asarray([i % 16], np.int32), one)
    print(f"latency {preset} {dtype}: {reps} single-request steps, latency rows/cluster {eng.latency_rows()}")
    eng.close()


def latency_trace(preset: str, reps: int, dtype: str) -> None:
    """Per-stage %globaltimer stamps of cluster rank 0 (thread 0) of each tower on
    the last of `reps` single-request steps, averaged per stage kind: each tower
    starts with input_up and input_down, then per block its layer's stages and the
    MLP's two (xLSTM six per block, the others five)."""
    import ctypes
    import os

    import numpy as np

    from . import build as B

    if not B.TRACE_LIB.exists():
        raise SystemExit(f"{B.TRACE_LIB} is missing: python -m hackathon_b200.build")
    os.environ["B2E_LIB"] = str(B.TRACE_LIB)
    from . import _lib
    from . import config as C
    from . import weights as W
    from .engine import EnsembleEngine

    cfg = C.PRESETS[preset]
    eng = EnsembleEngine(cfg, W.generate_model(cfg, 0), linear_dtype=dtype, capacity=16, max_batch=16)
    assert eng.latency_rows()[0] >= 1, "the latency path is off for this configuration"
    one = np.zeros((1, cfg.num_features), np.float32)
    for i in range(reps):
        eng.step(np.asarray([i % 16], np.int32), one)
    buf = np.zeros((4, 512, 8), np.uint64)
    rc = _lib.lib().b2e_lat_trace_read(ctypes.c_void_p(buf.ctypes.data))
    assert rc == 0, f"b2e_lat_trace_read: cudaError {rc}"
    eng.close()
    cols = ("cluster wait", "work", "next copies", "arrive")
    towers = ("xLSTM", "Mamba2", "RetNet", "Hawk")
    kinds = {0: ("A sLSTM", "B proj+qkv", "C mLSTM cell", "D down", "MLP1 fc1", "MLP2 fc2"),
             1: ("M1 proj+conv", "M2 ssm", "M3 out", "MLP1 fc1", "MLP2 fc2"),
             2: ("R1 proj+rotary", "R2 retention", "R3 out", "MLP1 fc1", "MLP2 fc2"),
             3: ("K1 proj+conv", "K2 rg-lru", "K3 out", "MLP1 fc1", "MLP2 fc2")}
    print(f"latency-trace {preset} {dtype}, one request, cluster rank 0; us per stage (bytes: the stage's copies)")
    for t in range(4):
        per = len(kinds[t])
        ns = 2 + cfg.tower_depth * per
        tr = buf[t, :ns].astype(np.int64)
        # fields: 0 start, 1 cluster barrier passed, 2 work done, 3 copies landed
        # (producer), 4 arrive issued, 5 arrived, 6 next stage's bytes
        d = np.stack([tr[:, 1] - tr[:, 0], tr[:, 2] - tr[:, 1], tr[:, 3] - tr[:, 1],
                      tr[:, 5] - tr[:, 4]], axis=1) / 1e3
        total = (tr[-1, 5] - tr[0, 0]) / 1e3
        print(f"{towers[t]}: {ns} stages, {total:.1f} us; mean " + ", ".join(f"{c} {d[:, i].mean():.2f}" for i, c in enumerate(cols)))
        for j in range(per):
            idx = [2 + b * per + j for b in range(cfg.tower_depth)]
            dd = d[idx].mean(axis=0)
            nb = float(np.mean(tr[[i - 1 for i in idx], 6]))
            print(f"  {kinds[t][j]:<16} " + "  ".join(f"{c} {dd[i]:5.2f}" for i, c in enumerate(cols)) + f"  bytes {nb:7.0f}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("cell")
    c.add_argument("--kind", required=True)
    c.add_argument("--rows", type=int, default=4096)
    c.add_argument("--heads", type=int, default=8)
    c.add_argument("--sh", type=int, default=64)
    c.add_argument("--sk", type=int, default=128)
    c.add_argument("--reps", type=int, default=4)
    c.add_argument("--waves", type=int, default=None, help="0: the step's persistent grid; default: the alone grid")
    li = sub.add_parser("linear")
    li.add_argument("--m", type=int, default=4096)
    li.add_argument("--k", type=int, default=512)
    li.add_argument("--n", type=int, default=256)
    li.add_argument("--reps", type=int, default=4)
    li.add_argument("--dtype", default="bf16")
    la = sub.add_parser("layer")
    la.add_argument("--kind", required=True)
    la.add_argument("--rows", type=int, default=4096)
    la.add_argument("--reps", type=int, default=4)
    la.add_argument("--dtype", default="bf16")
    la.add_argument("--micro", action="store_true", help="BASELINE config 2 / 3's layer (stated fills)")
    st = sub.add_parser("step")
    st.add_argument("--preset", default="D2")
    st.add_argument("--rows", type=int, default=2048)
    st.add_argument("--reps", type=int, default=4)
    st.add_argument("--dtype", default="bf16")
    lt = sub.add_parser("latency")
    lt.add_argument("--preset", default="D2")
    lt.add_argument("--reps", type=int, default=8)
    lt.add_argument("--dtype", default="bf16")
    lq = sub.add_parser("latency-trace")
    lq.add_argument("--preset", default="D2")
    lq.add_argument("--reps", type=int, default=30)
    lq.add_argument("--dtype", default="bf16")
    sub.add_parser("launches").add_argument("csv")
    sub.add_parser("metrics").add_argument("csv")
    a = ap.parse_args(argv)
    if a.cmd == "cell":
        cell(a.kind, a.rows, a.heads, a.sh, a.sk, a.reps, a.waves)
    elif a.cmd == "linear":
        linear(a.m, a.k, a.n, a.reps, a.dtype)
    elif a.cmd == "layer":
        layer(a.kind, a.rows, a.reps, a.dtype, a.micro)
    elif a.cmd == "step":
        step(a.preset, a.rows, a.reps, a.dtype)
    elif a.cmd == "latency":
        latency(a.preset, a.reps, a.dtype)
    elif a.cmd == "latency-trace":
        latency_trace(a.preset, a.reps, a.dtype)
    elif a.cmd == "launches":
        launches(a.csv)
    else:
        metrics(a.csv)


if __name__ == "__main__":
    main(sys.argv[1:])
