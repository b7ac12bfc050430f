"""Generate the golden fixtures by running the REFERENCE itself.

Runs only where the reference checkout is present (it is imported, never
copied): ``python tests/golden/make_golden.py --ref <reference checkout> <case>...``.
Every case loads the seeded weights of hackathon_b200.weights into the
reference's own torch modules (fp32, CPU), drives them through the reference's
own forward / masked-step / process_batch code, and stores what comes out as a
small .npz beside this script. The tests replay the same inputs through the CPU
oracle (oracle/) and the CUDA engine and compare.

Inputs are regenerated from seeds on both sides (numpy PCG64); each fixture
stores a checksum of its inputs so a generator drift fails loudly instead of
comparing different streams.

Cases
  cells      model/kernels.py *_reference on check_kernels.py's shapes and masks
  layers     the four layers of check_cell_rewrite.py's CASES, 12 masked steps
  model      MultiTowerModel at check_cell_rewrite.py's small config, masked steps,
             fp32 and with the reference's convert_linears (bf16 CastLinear)
  long       small model, 4 rows all active for 10,000 steps (long-stream drift)
  api        NnInferenceClient.process_batch at the small config: rounds, order,
             first-sight rows, capacity overflow answered with zeros
  d0stream   BASELINE config 1: default dims, 10,000 requests, SYM_001..SYM_016
             round-robin, one request per step (about 30 min on 8 cores)
  micro      BASELINE configs 2 and 3: the Mamba2, RetNet and xLSTM layers at
             their stated dims and fills, float32 and float64
  d0batch    BASELINE config 4: default dims, 256 symbols per step - its first 16
             rows, fp32 weights and the reference's bf16 CastLinear, 100 steps,
             and the first 4 rows in float64 (the arbiter)
  d0arbiter  the first 320 requests of d0stream through the reference model in
             float64 and in float32 (the arbiter of the fp32 D0 tolerance)
  d0emu      config 4's first 4 rows through the oracle's exact CastLinear bf16
             emulation (oracle/model.py, not the reference): a second correct bf16
             implementation, whose distance from the reference's bf16 run measures
             how far two such implementations drift apart over 100 steps
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from hackathon_b200 import config as C  # noqa: E402
from hackathon_b200 import weights as Wt  # noqa: E402
from tests.golden import streams  # noqa: E402

torch = None  # imported lazily with the reference


def _import_reference(ref: str):
    global torch
    import torch as _torch

    torch = _torch
    torch.set_num_threads(os.cpu_count() or 8)
    sys.path.insert(0, ref)
    import model.inference_model as im  # noqa: F401
    import model.kernels as kernels  # noqa: F401
    import model.mamba2, model.retnet, model.hawk, model.xlstm  # noqa: F401,E401

    return sys.modules


def _ref_cfg(mods, cfg: C.ModelConfig):
    im = mods["model.inference_model"]
    return im.ModelConfig(hidden_size=cfg.hidden_size, proj_size=cfg.proj_size,
                          tower_depth=cfg.tower_depth, num_heads=cfg.num_heads,
                          num_features=cfg.num_features)


def _load(module, sd):
    missing = module.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in sd.items()}, strict=True)
    del missing
    return module.eval()


def _leaves(state):
    if isinstance(state, (list, tuple)):
        for s in state:
            yield from _leaves(s)
    else:
        yield state


def _blend(old, new, mask):
    """The reference client's own fold (example_model.py:907-949)."""
    em = sys.modules.get("example_model")
    if em is None:
        import example_model as em  # noqa: F811
    holder = types.SimpleNamespace()
    holder._blend_state = types.MethodType(em.NnInferenceClient._blend_state, holder)
    holder._blend_state(old, new, mask)


def _save(name, meta, **arrays):
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, meta=np.array(json.dumps(meta)), **arrays)
    print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KiB)")


# ------------------------------------------------------------------ cases


def case_cells(mods):
    k = mods["model.kernels"]
    out = {}
    meta = {"cases": []}
    for tag, dims_list in streams.CELL_CASES.items():
        ref = {"mlstm": k.mlstm_step_reference, "retnet": k.retnet_step_reference,
               "mamba2": k.mamba2_step_reference}[tag]
        for ci, (batch, dims) in enumerate(dims_list):
            state0, rest, masks = streams.cell_inputs(tag, batch, dims, seed=100 + ci)
            for mname, mask in masks.items():
                st = torch.from_numpy(state0.copy())
                args = [torch.from_numpy(a) for a in rest]
                tm = None if mask is None else torch.from_numpy(mask)
                got = ref(st, *args, tm)
                key = f"{tag}_{ci}_{mname}"
                if mname == "mixed":  # all-true equals none; all-false leaves state0
                    out[f"{key}_state"] = st.numpy()
                out[f"{key}_out"] = got.numpy()
                meta["cases"].append({"key": key, "tag": tag, "batch": batch, "dims": list(dims),
                                      "seed": 100 + ci, "mask": mname})
    _save("cells", meta, **out)


def _layer_module(mods, tag, h):
    if tag == "xlstm":
        return mods["model.xlstm"].XLSTM(h, mlstm_num_heads=4, slstm_num_heads=2)
    if tag == "mamba2":
        return mods["model.mamba2"].Mamba2(h, head_size=16, bc_head_size=24)
    if tag == "retnet":
        return mods["model.retnet"].RetNet(h, num_heads=4)
    if tag == "hawk":
        return mods["model.hawk"].Hawk(h)
    raise ValueError(tag)


def case_layers(mods):
    out, meta = {}, {"cases": []}
    for tag, (cfg, steps, batch) in streams.LAYER_CASES.items():
        sd = Wt.generate(Wt.layer_specs(tag, "", cfg), seed=7)
        mod = _load(_layer_module(mods, tag, cfg.hidden_size), sd)
        xs, masks = streams.layer_stream(tag, cfg, steps, batch, seed=11)
        state = mod.init_state(batch, torch.device("cpu"))
        ys = []
        with torch.inference_mode():
            for s in range(steps):
                mask = torch.from_numpy(masks[s])
                y, new = mod(torch.from_numpy(xs[s]), state, mask=mask)
                _blend(state, new, mask)
                ys.append(y.numpy())
        out[f"{tag}_y"] = np.stack(ys)
        for i, leaf in enumerate(_leaves(state)):
            out[f"{tag}_state{i}"] = leaf.numpy()
        meta["cases"].append({"tag": tag, "steps": steps, "batch": batch, "weight_seed": 7,
                              "input_seed": 11, "input_sum": float(np.sum(xs, dtype=np.float64))})
    _save("layers", meta, **out)


def _model(mods, cfg, sd, lp=None):
    im = mods["model.inference_model"]
    m = _load(im.MultiTowerModel(_ref_cfg(mods, cfg)), sd)
    if lp is not None:
        import example_model as em

        em.convert_linears(m, {"bf16": torch.bfloat16, "fp16": torch.float16}[lp])
    return m


def case_model(mods):
    out, meta = {}, {"runs": []}
    cfg, steps, batch = streams.MODEL_CASE
    sd = Wt.generate_model(cfg, seed=0)
    feats, masks = streams.model_stream(cfg, steps, batch, seed=3)
    for lp in (None, "bf16"):
        m = _model(mods, cfg, sd, lp)
        state = m.init_state(batch, torch.device("cpu"))
        preds = []
        with torch.inference_mode():
            for s in range(steps):
                mask = torch.from_numpy(masks[s])
                p, new = m(torch.from_numpy(feats[s]), state, mask=mask)
                _blend(state, new, mask)
                preds.append(p.numpy())
        tag = lp or "fp32"
        out[f"{tag}_preds"] = np.stack(preds)
        for i, leaf in enumerate(_leaves(state)):
            out[f"{tag}_state{i}"] = leaf.numpy()
        meta["runs"].append(tag)
    meta.update({"steps": steps, "batch": batch, "weight_seed": 0, "input_seed": 3,
                 "input_sum": float(np.sum(feats, dtype=np.float64))})
    _save("model", meta, **out)


def case_long(mods):
    cfg, steps, batch = streams.LONG_CASE
    sd = Wt.generate_model(cfg, seed=0)
    m = _model(mods, cfg, sd)
    state = m.init_state(batch, torch.device("cpu"))
    gen = streams.long_features(cfg, batch, seed=5)
    preds = np.zeros((steps, batch, 4), np.float32)
    total = 0.0
    t0 = time.time()
    with torch.inference_mode():
        for s in range(steps):
            x = next(gen)
            total += float(np.sum(x, dtype=np.float64))
            p, state = m(torch.from_numpy(x), state)
            preds[s] = p.numpy()
    print(f"long: {steps} steps in {time.time() - t0:.0f} s")
    arrays = {"preds": preds}
    for i, leaf in enumerate(_leaves(state)):
        arrays[f"state{i}"] = leaf.numpy()
    _save("long", {"steps": steps, "batch": batch, "weight_seed": 0, "input_seed": 5,
                   "input_sum": total}, **arrays)


def case_api(mods, ref):
    import client as rclient
    import example_model as em

    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    sd_t = {k: torch.from_numpy(v) for k, v in sd.items()}
    em.hf_hub_download = lambda **kw: "<seeded>"
    real_load = torch.load
    torch.load = lambda f, **kw: sd_t if f == "<seeded>" else real_load(f, **kw)
    em.ModelConfig = lambda **kw: _ref_cfg(mods, cfg)  # the client hardcodes the default dims
    client = em.NnInferenceClient(num_symbols=streams.API_CAPACITY, device="cpu")
    calls = streams.api_calls(cfg)
    uids, preds, ncalls = [], [], []
    for call in calls:
        batch = {sym: [rclient.PendingRequest(unique_id=u, symbol=sym, features=f, received_time=0.0)
                       for (u, f) in reqs] for sym, reqs in call}
        r = client.process_batch(batch)
        uids += list(r.unique_ids)
        preds += [list(p) for p in r.predictions]
        ncalls.append(len(r.unique_ids))
    _save("api", {"capacity": streams.API_CAPACITY, "ncalls": ncalls,
                  "symbol_rows": client.symbol_to_idx},
          unique_ids=np.asarray(uids, np.int64), predictions=np.asarray(preds, np.float32))


def case_d0stream(mods, n_requests):
    cfg = C.D0
    sd = Wt.generate_model(cfg, seed=0)
    m = _model(mods, cfg, sd)
    del sd
    nsym = streams.D0_SYMBOLS
    states = [m.init_state(1, torch.device("cpu")) for _ in range(nsym)]
    feats = streams.d0_features(n_requests)
    preds = np.zeros((n_requests, 4), np.float32)
    t0 = time.time()
    with torch.inference_mode():
        for i in range(n_requests):
            s = i % nsym
            p, states[s] = m(torch.from_numpy(feats[i:i + 1]), states[s])
            preds[i] = p.numpy()[0]
            if i % 500 == 0:
                print(f"d0stream {i}/{n_requests} {time.time() - t0:.0f} s", flush=True)
    summ = {}
    for s in range(nsym):
        for li, leaf in enumerate(_leaves(states[s])):
            a = leaf.numpy().reshape(-1)
            summ[f"sym{s}_leaf{li}"] = streams.leaf_summary(a)
    _save("d0stream", {"n_requests": n_requests, "symbols": nsym, "weight_seed": 0,
                       "input_sum": float(np.sum(feats, dtype=np.float64))},
          preds=preds, **summ)


def case_d0batch(mods, steps):
    """BASELINE config 4 (default dims, 256 symbols, one request each per step) on
    its first D0_BATCH_ROWS rows - rows are independent, and the reference's step
    over all 256 needs more host memory than this machine has: the reference in
    float32 with fp32 weights and with its own convert_linears to bf16, `steps`
    steps from zero state; predictions per step and per-leaf state summaries of
    the first row at the end."""
    cfg = C.D0
    sd = Wt.generate_model(cfg, seed=0)
    rows = streams.D0_BATCH_ROWS
    out = {}
    for lp in (None, "bf16"):
        m = _model(mods, cfg, sd, lp)
        state = m.init_state(rows, torch.device("cpu"))
        preds = np.zeros((steps, rows, 4), np.float32)
        t0 = time.time()
        with torch.inference_mode():
            for s in range(steps):
                x = streams.d0_batch_features(s)[:rows]
                p, state = m(torch.from_numpy(x), state)
                preds[s] = p.float().numpy()
                if s % 10 == 0:
                    print(f"d0batch {lp or 'fp32'} {s}/{steps} {time.time() - t0:.0f} s", flush=True)
        tag = lp or "fp32"
        out[f"{tag}_preds"] = preds
        for li, leaf in enumerate(_leaves(state)):
            out[f"{tag}_row0_leaf{li}"] = streams.leaf_summary(leaf[0].float().numpy() if leaf.is_floating_point()
                                                               else leaf[0].numpy())
        del m, state
    # the float64 arbiter on the first D0_BATCH_ARBITER rows (weights and state in double)
    m = _model(mods, cfg, sd).to(torch.float64)
    ra = streams.D0_BATCH_ARBITER
    state = _cast_state(m.init_state(ra, torch.device("cpu")), torch.float64)
    preds = np.zeros((steps, ra, 4), np.float64)
    t0 = time.time()
    with torch.inference_mode():
        for s in range(steps):
            x = torch.from_numpy(streams.d0_batch_features(s)[:ra]).to(torch.float64)
            p, state = m(x, state)
            preds[s] = p.numpy()
            if s % 10 == 0:
                print(f"d0batch f64 {s}/{steps} {time.time() - t0:.0f} s", flush=True)
    out["f64_preds"] = preds
    del m, state
    _save("d0batch", {"steps": steps, "rows": rows, "arbiter_rows": ra, "weight_seed": 0}, **out)


def case_d0emu(steps):
    """The oracle's bf16 CastLinear emulation (input and weights rounded to bf16,
    float32 accumulation, one rounding of the sum) on config 4's arbiter rows."""
    from oracle import model as O

    cfg = C.D0
    sd = Wt.generate_model(cfg, seed=0)
    ra = streams.D0_BATCH_ARBITER
    # the oracle rounds a weight to bf16 on every call; the weight matrices (the
    # only arrays of a million elements or more here) are rounded once instead
    lowp, memo = O.lowp, {}

    def lowp_once(a, lp):
        if a.size < (1 << 20):
            return lowp(a, lp)
        key = (id(a), lp)
        if key not in memo:
            memo[key] = lowp(a, lp)
        return memo[key]

    O.lowp = lowp_once
    orc = O.Oracle(cfg, sd, lp="bf16")
    st = O.init_state(cfg, ra)
    preds = np.zeros((steps, ra, 4), np.float32)
    t0 = time.time()
    for s in range(steps):
        p, st = orc.step(streams.d0_batch_features(s)[:ra], st)
        preds[s] = p
        if s % 10 == 0:
            print(f"d0emu {s}/{steps} {time.time() - t0:.0f} s", flush=True)
    O.lowp = lowp
    _save("d0batch_emu", {"steps": steps, "rows": ra, "weight_seed": 0,
                          "source": "oracle/model.py Oracle(lp='bf16'), not the reference"}, emu_preds=preds)


def case_d0arbiter(mods, n_requests):
    """The first n_requests of BASELINE config 1 through the reference's model in
    float64 (same seeded weights, module and state in double) and again in
    float32: the float64 run is the arbiter that measures how far each fp32
    implementation (the reference's torch CPU path, the CUDA engine) is from the
    exact answer."""
    cfg = C.D0
    sd = Wt.generate_model(cfg, seed=0)
    nsym = streams.D0_SYMBOLS
    feats = streams.d0_features(n_requests)
    out = {}
    for tag, dt in (("f64", torch.float64), ("f32", torch.float32)):
        m = _model(mods, cfg, sd).to(dt)
        states = [m.init_state(1, torch.device("cpu")) for _ in range(nsym)]
        states = [_cast_state(st, dt) for st in states]
        preds = np.zeros((n_requests, 4), np.float64)
        t0 = time.time()
        with torch.inference_mode():
            for i in range(n_requests):
                k = i % nsym
                p, states[k] = m(torch.from_numpy(feats[i:i + 1]).to(dt), states[k])
                preds[i] = p.double().numpy()[0]
                if i % 50 == 0:
                    print(f"d0arbiter {tag} {i}/{n_requests} {time.time() - t0:.0f} s", flush=True)
        out[f"{tag}_preds"] = preds
        for k in range(nsym):
            for li, leaf in enumerate(_leaves(states[k])):
                a = leaf.double().numpy().reshape(-1) if leaf.is_floating_point() else leaf.numpy().reshape(-1)
                out[f"{tag}_sym{k}_leaf{li}"] = streams.leaf_summary(a)
        del m, states
    _save("d0arbiter", {"n_requests": n_requests, "symbols": nsym, "weight_seed": 0,
                        "input_sum": float(np.sum(feats, dtype=np.float64))}, **out)


def case_micro(mods):
    """BASELINE configs 2 and 3: Mamba2(256, head 64, d_state 64) with its stated
    a / dt fills, RetNet(256, 4 heads of 64) with gamma_h = 1 - 2^(-5-h), and
    XLSTM(128, 4 mLSTM heads of 64), each over MICRO_STEPS steps of MICRO_BATCH
    rows (all active), in float32 and in float64 (the arbiter)."""
    out, meta = {}, {"cases": []}
    for kind in ("mamba2", "retnet", "xlstm"):
        cfg, sd = Wt.micro_layer(kind, seed=0)
        xs = streams.micro_inputs(kind)
        for tag, dt in (("f32", torch.float32), ("f64", torch.float64)):
            if kind == "mamba2":
                mod = mods["model.mamba2"].Mamba2(cfg.hidden_size, head_size=cfg.mamba_head_size,
                                                  bc_head_size=cfg.mamba_bc_size)
            elif kind == "retnet":
                mod = mods["model.retnet"].RetNet(cfg.hidden_size, num_heads=cfg.num_heads)
            else:
                mod = mods["model.xlstm"].XLSTM(cfg.hidden_size, mlstm_num_heads=cfg.num_heads,
                                                slstm_num_heads=cfg.num_heads // 2)
            mod = _load(mod, sd).to(dt)
            state = _cast_state(mod.init_state(xs.shape[1], torch.device("cpu")), dt)
            ys = []
            with torch.inference_mode():
                for s in range(xs.shape[0]):
                    y, state = mod(torch.from_numpy(xs[s]).to(dt), state)
                    ys.append(y.float().numpy())
            # float64 results are stored rounded to float32: 6e-8 relative, far
            # below the fp32 rounding noise (1e-6 and up) they arbitrate
            out[f"{kind}_{tag}_y"] = np.stack(ys)
            for i, leaf in enumerate(_leaves(state)):
                out[f"{kind}_{tag}_state{i}"] = leaf.float().numpy() if leaf.is_floating_point() else leaf.numpy()
        meta["cases"].append({"kind": kind, "steps": int(xs.shape[0]), "batch": int(xs.shape[1]),
                              "input_sum": float(np.sum(xs, dtype=np.float64))})
    _save("micro", meta, **out)


def _cast_state(state, dt):
    if isinstance(state, (list, tuple)):
        return type(state)(_cast_state(s, dt) for s in state)
    return state.to(dt) if state.is_floating_point() else state


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("cases", nargs="+")
    ap.add_argument("--d0-requests", type=int, default=10_000)
    ap.add_argument("--arbiter-requests", type=int, default=320)
    ap.add_argument("--d0batch-steps", type=int, default=100)
    a = ap.parse_args()
    mods = _import_reference(a.ref)
    for c in a.cases:
        t = time.time()
        if c == "cells":
            case_cells(mods)
        elif c == "layers":
            case_layers(mods)
        elif c == "model":
            case_model(mods)
        elif c == "long":
            case_long(mods)
        elif c == "api":
            case_api(mods, a.ref)
        elif c == "d0stream":
            case_d0stream(mods, a.d0_requests)
        elif c == "micro":
            case_micro(mods)
        elif c == "d0batch":
            case_d0batch(mods, a.d0batch_steps)
        elif c == "d0emu":
            case_d0emu(a.d0batch_steps)
        elif c == "d0arbiter":
            case_d0arbiter(mods, a.arbiter_requests)
        else:
            raise SystemExit(f"unknown case {c}")
        print(f"{c}: {time.time() - t:.0f} s")


if __name__ == "__main__":
    main()
