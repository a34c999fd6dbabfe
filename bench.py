#!/usr/bin/env python
"""Benchmark of the IFKFAC curvature hot path on B200.

One step = one single-layer operator: streaming TSQR of X and delta
(16384 x 4096 bf16 each, 8 row tiles of 2048 folded one after another into
R_X / R_G), the damping fold (R/sqrt(p), lambda = 1e-2) to bf16 factors, the
four triangular solves on grad_W (4096 x 4096 fp32) and the momentum 0.9 /
lr 1e-3 update of fp32 master weights.  Inputs are synthetic with the
config's distributions (no dataset is involved): X, delta ~ N(0,1) times
per-column scales log-uniform in [1, 100] (kappa ~ 1e2), grad_W ~ N(0, 1e-2).

Fold schedules (--schedule), both with the reflector sequence of the streaming
fold, one 256-row sub-tile after another in tile order, and the same factors:
  one-launch (default): the tiles are resident, so one persistent launch per
      step folds all of them in order together with the damping rows
      sqrt(lambda p) I, and the result is scaled by 1/sqrt(p) (exact for
      p = 16384, a power of 4);
  per-tile: one fold launch per tile as it would arrive from a hook, then the
      damping fold.
The other schedule is timed too and reported as "other_schedule".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (launched with torchrun, one rank per GPU): layers are dealt
round-robin to ranks (rank r owns layer r with its own data), so the units
are independent and no collective is on the data path ("scaling": "weak");
timing is the max over ranks of the device-timed region.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_DIM, P_ROWS, TILE, DAMPING, LR, MOM = 4096, 16384, 2048, 1e-2, 1e-3, 0.9
METRIC = "preconditioned steps/sec; TSQR+trsm TFLOP/s on 4096² bf16 layer, 1/2/4/8 B200"
WORKLOAD = ("C2 single-layer operator: streaming TSQR of X and delta (16384x4096 bf16, 8 tiles of 2048), "
            "damping fold lambda=1e-2 to bf16 R, 4 trsm on grad_W 4096x4096 fp32, momentum/lr update")


def algorithmic_flops(n=N_DIM, p=P_ROWS, n_in=N_DIM, n_out=N_DIM):
    """Algorithmic work of one operator (extra flops of an implementation do not count):
    TSQR 2*(2pn^2 - 2/3 n^3), two triangle-on-diagonal damping folds 2*(2/3 n^3),
    four trsm 2*n_out^2*n_in + 2*n_in^2*n_out."""
    tsqr = 2 * (2 * p * n * n - 2.0 / 3.0 * n ** 3)
    fold = 2 * (2.0 / 3.0 * n ** 3)
    trsm = 2 * n_out * n_out * n_in + 2 * n_in * n_in * n_out
    return {"tsqr": tsqr, "fold": fold, "trsm": trsm, "tsqr_fold": tsqr + fold, "total": tsqr + fold + trsm}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "hbm": d["hbm_gbs"], "source": "measured"}
    except Exception:
        return {"bf16": 1590.0, "bf16_sustained": 1400.0, "hbm": 6650.0, "source": "fallback"}


def graph_kernel_names(graph):
    """Kernel names of the nodes of a captured torch CUDA graph (driver-API introspection)."""
    import cuda.bindings.driver as drv
    g = drv.CUgraph(graph.raw_cuda_graph())
    err, _, n = drv.cuGraphGetNodes(g, 0)
    err, nodes, n = drv.cuGraphGetNodes(g, n)
    names = []
    for nd in nodes[:n]:
        err, t = drv.cuGraphNodeGetType(nd)
        if t != drv.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
            continue
        err, prm = drv.cuGraphKernelNodeGetParams(nd)
        err, name = drv.cuFuncGetName(prm.func)
        names.append(name.decode() if isinstance(name, bytes) else str(name))
    return names


def count_launches(graph):
    """libifk kernels (namespace ifk) per captured step, and the other kernels in it."""
    try:
        names = graph_kernel_names(graph)
    except Exception as e:  # introspection unavailable: report it instead of guessing
        return None, None, f"graph introspection failed: {type(e).__name__}"
    ours = [n for n in names if "3ifk" in n]
    return len(ours), len(names) - len(ours), "kernel nodes of the captured step graph"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # the timed region starts once the sampler answers (its start-up takes a moment)
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.01)
            self.lines.clear()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1].split()[0]))
                mx = float(f[2].split()[0])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz)}


def make_inputs(device, seed):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)

    def scaled():
        s = torch.exp(torch.rand(N_DIM, generator=g, device=device) * math.log(100.0))
        return (torch.randn(P_ROWS, N_DIM, generator=g, device=device) * s).to(torch.bfloat16)

    X, D = scaled(), scaled()
    gW = torch.randn(N_DIM, N_DIM, generator=g, device=device) * 1e-2
    W = torch.randn(N_DIM, N_DIM, generator=g, device=device) * 1e-2
    return X, D, gW, W


def make_layer(dev, per_tile, ntiles):
    """Device state of the layer: fp32 running factors, bf16 damped factors."""
    from ifkfac_b200 import _lib
    from ifkfac_b200.engine import LayerCurvature
    import torch
    return LayerCurvature(N_DIM, N_DIM, dev, _lib.PREC_BF16, torch.bfloat16, TILE,
                          window=1 if per_tile else ntiles)


def run_step(lc, per_tile, tiles, x, d, g, w):
    """One operator step.  Schedules (same reflector sequence, same factors):
    "one-launch": the row tiles are resident, so they are folded in arrival order
    by one persistent launch per factor pair together with the damping rows
    (ifk_tsqr_fold_segments with an identity tail), then scaled by 1/sqrt(p);
    "per-tile": one fold launch per tile as it arrives, then the damping fold."""
    lc.clear()
    for lo, hi in tiles:
        lc.fold(x[lo:hi], d[lo:hi])
    lc.refresh(DAMPING, consume=not per_tile)
    lc.natgrad_update(g, w, LR, MOM)


def time_components(lc, per_tile, tiles, X, D, gW, W):
    """Device time of each stage of one eager step (CUDA events on the launching stream)."""
    import torch
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def timed(fn):
        a, b = ev(), ev()
        a.record()
        fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b)

    lc.clear()
    torch.cuda.synchronize()
    comp = {}
    if per_tile:
        comp["tsqr_ms"] = sum(timed(lambda: lc.fold(X[lo:hi], D[lo:hi])) for lo, hi in tiles)
        comp["fold_ms"] = timed(lambda: lc.refresh(DAMPING))
    else:
        for lo, hi in tiles:
            lc.fold(X[lo:hi], D[lo:hi])  # kept for the launch below: no device work
        comp["tsqr_fold_ms"] = timed(lambda: lc.refresh(DAMPING, consume=True))
    # the step's natural gradient + update (one call; the last solve applies the update)
    comp["trsm_update_ms"] = timed(lambda: lc.natgrad_update(gW, W, LR, MOM))
    # the two halves as separate calls, for reference
    nat = [None]

    def nat_fn():
        nat[0] = lc.natgrad(gW)

    comp["trsm_ms"] = timed(nat_fn)
    comp["update_ms"] = timed(lambda: lc.update(W, nat[0], LR, MOM, 0.0, None))
    return comp


def time_fp32_mode(dev, X, D, gW, W, tiles):
    """The same operator in the fp32 mode (IFK_PREC_FP32, the reference's
    use_true_bf16=False path at its 1e-5 bound): fp32 rows, the one-launch schedule
    like the headline (the 8 tiles of both factors through one wave schedule, then
    the damping rows; fp32 Householder panels, fp32 trailing updates on the CUDA
    cores), fp32 factors, fp32 solves and the update.  Timed as a CUDA graph of the step
    (CUDA events, one GPU); the component split is one eager step."""
    import torch
    from ifkfac_b200 import _lib
    from ifkfac_b200.engine import LayerCurvature
    lc = LayerCurvature(N_DIM, N_DIM, dev, _lib.PREC_FP32, torch.float32, TILE, window=len(tiles))
    Xf, Df, Wf = X.float(), D.float(), W.clone()
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def step(comp=None, marked=True):
        marks = [ev() for _ in range(4)] if marked else None
        mark = (lambda i: marks[i].record()) if marked else (lambda i: None)
        mark(0)
        lc.clear()
        for lo, hi in tiles:
            lc.fold(Xf[lo:hi], Df[lo:hi])
        mark(1)
        lc.refresh(DAMPING, consume=True)
        mark(2)
        lc.natgrad_update(gW, Wf, LR, MOM)
        mark(3)
        if comp is not None:
            marks[3].synchronize()
            # the tiles are kept by fold() and folded with the damping rows by refresh()
            comp.update(tsqr_fold_ms=marks[0].elapsed_time(marks[2]),
                        trsm_update_ms=marks[2].elapsed_time(marks[3]))

    step()
    torch.cuda.synchronize()
    comp = {}
    step(comp)
    # the step captured in a CUDA graph, like the headline's (its fp32 solves are
    # many short launches); eager if the capture fails
    graph, timing = None, "eager, CUDA events, one GPU"
    try:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step(marked=False)
        torch.cuda.current_stream().wait_stream(s)
        with torch.cuda.graph(g, stream=s):
            step(marked=False)
        g.replay()
        torch.cuda.synchronize()
        graph, timing = g, "CUDA graph of the step, CUDA events, one GPU (components: one eager step)"
    except Exception as e:  # noqa: BLE001 - reported in the line
        timing = f"eager, CUDA events, one GPU (graph capture failed: {type(e).__name__})"
    k = 3
    a, b = ev(), ev()
    a.record()
    for _ in range(k):
        if graph is not None:
            graph.replay()
        else:
            step(marked=False)
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / k
    out = {"ms_per_step": ms, "value": 1000.0 / ms, "unit": "steps/s", "dtype": "f32",
           "timing": timing, "components_ms": comp}
    del graph
    del lc, Xf, Df, Wf
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world, local_rank):
    import torch
    from ifkfac_b200 import _lib
    from ifkfac_b200.engine import LayerCurvature

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    _lib.check(_lib.lib().ifk_device_check(), "ifk_device_check")
    X, D, gW, W = make_inputs(dev, 1234 + rank)
    tiles = [(t * TILE, (t + 1) * TILE) for t in range(P_ROWS // TILE)]
    per_tile = args.schedule == "per-tile"
    lc = make_layer(dev, per_tile, len(tiles))

    def step(x, d, g, w):
        run_step(lc, per_tile, tiles, x, d, g, w)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # warm-up (also sets kernel attributes and creates the momentum buffer)
    for _ in range(args.warmup):
        step(X, D, gW, W)
    torch.cuda.synchronize()
    if args.profile:
        # one eager step for a profiler's launch list; no timing, no output line
        torch.cuda.nvtx.range_push("ifk_profile_step")
        step(X, D, gW, W)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        return
    graph = None
    if True:
        # the step graph is timed unless --no-graph; it is always captured to count launches
        graph = torch.cuda.CUDAGraph(keep_graph=True)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step(X, D, gW, W)  # one more eager warm-up on the capture stream
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=s):
                step(X, D, gW, W)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph.instantiate()
        graph.replay()
        torch.cuda.synchronize()

    n_ours, n_other, launch_src = count_launches(graph)
    if args.no_graph:
        graph = None

    def run_steps(k):
        for _ in range(k):
            if graph is not None:
                graph.replay()
            else:
                step(X, D, gW, W)

    # ---- timed region: device time, max over ranks ----
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e0.record()
        run_steps(args.steps)
        e1.record()
        e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    flops = algorithmic_flops()
    pk = peaks()

    # ---- component timing (eager, events on the launching stream) ----
    comp = {}
    if rank == 0:
        comp = time_components(lc, per_tile, tiles, X, D, gW, W)

    # ---- secondary: the other schedule of the same step (eager timing) ----
    other = None
    if rank == 0 and not args.no_other_schedule:
        lco = make_layer(dev, not per_tile, len(tiles))
        Wo = W.clone()
        for _ in range(2):
            run_step(lco, not per_tile, tiles, X, D, gW, Wo)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ko = max(1, min(args.steps, 5))
        a.record()
        for _ in range(ko):
            run_step(lco, not per_tile, tiles, X, D, gW, Wo)
        b.record()
        b.synchronize()
        oms = a.elapsed_time(b) / ko
        other = {"schedule": "one-launch" if per_tile else "per-tile", "ms_per_step": oms,
                 "value": 1000.0 / oms, "unit": "steps/s", "timing": "eager, CUDA events, one GPU",
                 "components_ms": time_components(lco, not per_tile, tiles, X, D, gW, Wo)}
        del lco, Wo

    # ---- secondary: the fp32 mode (use_true_bf16=False) on the same operator ----
    fp32 = None
    if rank == 0 and not args.no_fp32_mode:
        fp32 = time_fp32_mode(dev, X, D, gW, W, tiles)

    # ---- end to end through the public API: pinned host inputs in, weights out ----
    e2e = None
    if rank == 0 or world > 1:
        hX = X.cpu().pin_memory()
        hD = D.cpu().pin_memory()
        hG = gW.cpu().pin_memory()
        hW = torch.empty_like(W, device="cpu").pin_memory()
        bi = hX.numel() * 2 + hD.numel() * 2 + hG.numel() * 4
        bo = hW.numel() * 4
        k2 = max(2, min(args.steps, 10))
        # Every step copies all of its inputs from pinned host memory and reads the
        # updated W back.  The device inputs are double-buffered, so the copies of
        # step k + 1 (on a copy stream) run under the compute of step k, and the
        # read-back of W runs on its own stream (the next update waits for it).
        # per-tile: the fold of a tile waits for that tile only.  one-launch: the
        # tiles are folded in --e2e-groups launches of consecutive tiles (the last
        # one with the damping rows), each waiting for its own tiles.
        cs, dh = torch.cuda.Stream(), torch.cuda.Stream()
        s0 = torch.cuda.current_stream()
        if per_tile:
            sizes = [len(tiles)]
        else:
            sizes = [int(x) for x in str(args.e2e_groups).split(",") if int(x) > 0]
            if len(sizes) == 1:  # a count of equal groups
                ng = max(1, min(sizes[0], len(tiles)))
                sizes = [round((i + 1) * len(tiles) / ng) - round(i * len(tiles) / ng) for i in range(ng)]
            if sum(sizes) != len(tiles):
                raise SystemExit(f"--e2e-groups {args.e2e_groups}: group sizes must add up to {len(tiles)} tiles")
        ng = len(sizes)
        bounds = [sum(sizes[:i]) for i in range(ng + 1)]
        bufs = [(X, D, gW), (torch.empty_like(X), torch.empty_like(D), torch.empty_like(gW))]
        st = {"free": [None, None], "wdone": None, "k": 0}

        def e2e_step():
            xb, db, gb = bufs[st["k"] % 2]
            evs = []
            with torch.cuda.stream(cs):
                if st["free"][st["k"] % 2] is not None:
                    cs.wait_event(st["free"][st["k"] % 2])  # step k - 2 is done reading this buffer
                for lo, hi in tiles:
                    xb[lo:hi].copy_(hX[lo:hi], non_blocking=True)
                    db[lo:hi].copy_(hD[lo:hi], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(cs)
                    evs.append(e)
                gb.copy_(hG, non_blocking=True)
                eg = torch.cuda.Event()
                eg.record(cs)
            lc.clear()
            if per_tile:
                for (lo, hi), e in zip(tiles, evs):
                    s0.wait_event(e)
                    lc.fold(xb[lo:hi], db[lo:hi])
                lc.refresh(DAMPING)
            else:
                for gi in range(ng):
                    s0.wait_event(evs[bounds[gi + 1] - 1])
                    for lo, hi in tiles[bounds[gi]:bounds[gi + 1]]:
                        lc.fold(xb[lo:hi], db[lo:hi])
                    if gi + 1 < ng:
                        lc.flush()
                lc.refresh(DAMPING, consume=True)
            s0.wait_event(eg)
            if st["wdone"] is not None:
                s0.wait_event(st["wdone"])  # the previous read-back of W has finished
            lc.natgrad_update(gb, W, LR, MOM)
            fe = torch.cuda.Event()
            fe.record(s0)
            st["free"][st["k"] % 2] = fe
            ue = torch.cuda.Event()
            ue.record(s0)
            dh.wait_event(ue)
            with torch.cuda.stream(dh):
                hW.copy_(W, non_blocking=True)
                wd = torch.cuda.Event()
                wd.record(dh)
            st["wdone"] = wd
            st["k"] += 1

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k2):
            e2e_step()
        s0.wait_event(st["wdone"])  # the last step's W is on the host
        b.record()
        b.synchronize()
        e2e_ms = a.elapsed_time(b) / k2
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": world * 1000.0 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": bi,
               "d2h_bytes_per_step": bo, "ms_per_step": e2e_ms,
               "schedule": args.schedule, "launch_groups": sizes,
               "note": ("every step copies its X, delta (per tile) and grad_W from pinned host memory and reads "
                        "the updated W back; device inputs double-buffered, so step k+1's copies run under step "
                        "k's compute; each fold launch waits for its own tiles only")}

    if rank != 0:
        return
    out = {
        "metric": METRIC, "value": world * 1000.0 / ms, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "n": N_DIM, "p": P_ROWS, "tile_rows": TILE,
                   "damping": DAMPING, "lr": LR, "momentum": MOM, "use_true_bf16": True,
                   "parallelism": f"layers round-robin over {world} GPU(s)",
                   "l2": "inputs larger than L2 (X + delta bf16 = 268 MB read per step)",
                   "cuda_graph": graph is not None},
        "tflops": world * flops["total"] / (ms * 1e-3) / 1e12,
        "tflops_frac_of_measured_bf16": flops["total"] / (ms * 1e-3) / 1e12 / pk["bf16"],
        "components_ms": comp,
        "schedule": args.schedule,
        "other_schedule": other,
        "fp32_mode": fp32,
        "gpu_launches": (n_ours * args.steps) if n_ours is not None else None,
        "gpu_launches_detail": {"libifk_per_step": n_ours, "torch_per_step": n_other, "source": launch_src},
        "clocks": clk.summary(),
        "e2e": e2e,
    }
    if comp:
        # dominant component by time; achieved = its algorithmic flops / its device time
        stages = [("tsqr_fold", "tsqr_fold_ms"), ("tsqr", "tsqr_ms"), ("fold", "fold_ms"), ("trsm", "trsm_ms")]
        name, key = max(((nm, k) for nm, k in stages if k in comp), key=lambda x: comp[x[1]])
        ach = flops[name] / (comp[key] * 1e-3) / 1e12
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
                traffic = json.load(f).get(name)
        except Exception:
            pass
        out["roofline"] = {"kernel": f"{name} (all libifk launches of the {name} stage, one step)",
                           "bound": "tensor", "achieved": ach, "peak": pk["bf16"],
                           "unit": "TFLOP/s", "frac": ach / pk["bf16"], "traffic": traffic,
                           "peak_source": f"{pk['source']} bf16 burst"}
    if not args.no_cpu_baseline and world == 1:
        out["cpu_baseline"] = cpu_baseline()
    print(json.dumps(out), flush=True)


def run_sharded(args, rank, world, local_rank):
    """Config 2 on N GPUs with the path's own partition: the same single-layer operator
    at every N (strong scaling).  The 16384 rows of X and delta are batch-sharded, p / N
    per rank; every rank folds its rows into local factors (rank 0 with the damping rows
    sqrt(lambda p) I as the last segment of the same launch); the local factors are
    combined by the R-tree of the reference's tsqr (ifkfac/triangular.py:207-220):
    ceil(log2 N) rounds of pairwise NCCL send / recv, both factors of a round merged in
    one launch (trapezoidal-chunk folds); the owner of the layer (rank 0) finalises
    (1 / sqrt(p), bf16 cast), runs the four solves with the fused momentum / lr update
    and broadcasts W to every rank.  Timing: K eager steps between barriers, CUDA events,
    max over ranks; the per-stage split is taken on every rank and gathered."""
    import ctypes
    import torch
    import torch.distributed as dist
    from ifkfac_b200 import _lib
    from ifkfac_b200.engine import LayerCurvature, fold_segments, _arr, _ws

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L = _lib.lib()
    _lib.check(L.ifk_device_check(), "ifk_device_check")
    X, D, gW, W = make_inputs(dev, 1234)  # the same operator on every rank
    rows = P_ROWS // world
    lo = rank * rows
    tiles = [(a, min(a + TILE, lo + rows)) for a in range(lo, lo + rows, TILE)]
    lc = LayerCurvature(N_DIM, N_DIM, dev, _lib.PREC_BF16, torch.bfloat16, TILE, window=len(tiles))
    fx, fg = lc.fx, lc.fg
    other = [torch.empty(N_DIM, N_DIM, device=dev), torch.empty(N_DIM, N_DIM, device=dev)]
    ws_m = _ws(L.ifk_tsqr_fold_batched_workspace(2, _arr(ctypes.c_int64, [N_DIM, N_DIM]),
                                                  _arr(ctypes.c_int64, [N_DIM, N_DIM])), dev)
    stream = lambda: torch.cuda.current_stream().cuda_stream
    # rows of each rank's local factor (rank 0 holds the damping rows too)
    local_rows = [min(N_DIM, rows + (N_DIM if r == 0 else 0)) for r in range(world)]
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def merge_into(rb):
        n2 = _arr(ctypes.c_int64, [N_DIM, N_DIM])
        _lib.check(L.ifk_tsqr_fold_batched(
            2, _arr(ctypes.c_void_p, [fx.R.data_ptr(), fg.R.data_ptr()]), n2,
            _arr(ctypes.c_int64, [fx.rows_R, fg.rows_R]),
            _arr(ctypes.c_void_p, [other[0].data_ptr(), other[1].data_ptr()]), n2,
            _arr(ctypes.c_int64, [rb, rb]), n2, _lib.F32, _lib.PREC_BF16, _lib.FOLD_TRAPEZOIDAL_CHUNK,
            lc.status.data_ptr(), ws_m.data_ptr(), ws_m.numel(), stream()), "ifk_tsqr_fold_batched")
        fx.rows_R = fg.rows_R = min(N_DIM, fx.rows_R + rb)

    def step(marks=None):
        mark = (lambda: marks.append(ev()) or marks[-1].record()) if marks is not None else (lambda: None)
        mark()
        lc.clear()
        segs = ([X[a:b] for a, b in tiles], [D[a:b] for a, b in tiles])
        tails = [math.sqrt(DAMPING * P_ROWS)] * 2 if rank == 0 else None
        lc.ws_pair = fold_segments((fx, fg), segs, lc.ws_pair, ident_tail=tails)
        fx.consumed = fg.consumed = False  # merged below, then finalised; cleared next step
        mark()
        s = 1
        while s < world:
            if rank % (2 * s) == 0:
                partner = rank + s
                if partner < world:
                    rb = min(N_DIM, sum(local_rows[partner:partner + s]))
                    for w in dist.batch_isend_irecv([dist.P2POp(dist.irecv, other[0], partner),
                                                     dist.P2POp(dist.irecv, other[1], partner)]):
                        w.wait()
                    merge_into(rb)
            else:
                for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, fx.R, rank - s),
                                                 dist.P2POp(dist.isend, fg.R, rank - s)]):
                    w.wait()
                break
            s *= 2
        mark()
        if rank == 0:
            _lib.check(L.ifk_finalize_batched(
                2, _arr(ctypes.c_void_p, [fx.R.data_ptr(), fg.R.data_ptr()]), _arr(ctypes.c_int64, [N_DIM] * 2),
                _arr(ctypes.c_int64, [fx.rows_R, fg.rows_R]), _arr(ctypes.c_int64, [N_DIM] * 2),
                _arr(ctypes.c_double, [float(P_ROWS)] * 2), 0.0,
                _arr(ctypes.c_void_p, [lc.RX.data_ptr(), lc.RG.data_ptr()]), _arr(ctypes.c_int64, [N_DIM] * 2),
                _lib.BF16, _lib.PREC_BF16, lc.status.data_ptr(), lc.ws_fin.data_ptr(), lc.ws_fin.numel(),
                stream()), "ifk_finalize_batched")
            lc.natgrad_update(gW, W, LR, MOM)
        mark()
        dist.broadcast(W, src=0)
        mark()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # per-stage split of one step on every rank (eager, events on the launching stream)
    marks = []
    dist.barrier()
    step(marks)
    torch.cuda.synchronize()
    names = ["local_fold", "rtree_merge", "finalize_solve_update", "broadcast_W"]
    mine = torch.tensor([marks[i].elapsed_time(marks[i + 1]) for i in range(len(names))], device=dev)
    allst = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allst, mine)
    # timed region
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    with ClockSampler(local_rank) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        e1.synchronize()
    dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # end to end: each rank's rows (and rank 0's grad_W) from pinned host memory every
    # step, W read back to the host by rank 0
    hX = X[lo:lo + rows].cpu().pin_memory()
    hD = D[lo:lo + rows].cpu().pin_memory()
    hG = gW.cpu().pin_memory()
    hW = torch.empty_like(W, device="cpu").pin_memory()

    def e2e_step():
        X[lo:lo + rows].copy_(hX, non_blocking=True)
        D[lo:lo + rows].copy_(hD, non_blocking=True)
        if rank == 0:
            gW.copy_(hG, non_blocking=True)
        step()
        if rank == 0:
            hW.copy_(W, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    k2 = max(2, min(args.steps, 10))
    a, b = ev(), ev()
    a.record()
    for _ in range(k2):
        e2e_step()
    b.record()
    b.synchronize()
    e2e_ms = a.elapsed_time(b) / k2
    t = torch.tensor([e2e_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    if rank != 0:
        return
    flops = algorithmic_flops()
    pk = peaks()
    stages = {nm: [float(x[i]) for x in allst] for i, nm in enumerate(names)}
    out = {
        "metric": METRIC, "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "n": N_DIM, "p": P_ROWS, "tile_rows": TILE, "damping": DAMPING,
                   "lr": LR, "momentum": MOM, "use_true_bf16": True,
                   "parallelism": (f"rows batch-sharded over {world} GPUs ({rows} each), R-tree over NCCL "
                                   "send/recv, solves + update on the layer's owner, W broadcast"),
                   "l2": "inputs larger than L2 (X + delta bf16 = 268 MB read per step)", "cuda_graph": False},
        "tflops": flops["total"] / (ms * 1e-3) / 1e12,
        "tflops_frac_of_measured_bf16": flops["total"] / (ms * 1e-3) / 1e12 / pk["bf16"],
        "stages_ms_per_rank": stages,
        "clocks": clk.summary(),
        "e2e": {"value": 1000.0 / e2e_ms, "unit": "steps/s",
                "h2d_bytes_per_step": X.numel() * 2 + D.numel() * 2 + gW.numel() * 4,
                "d2h_bytes_per_step": W.numel() * 4, "ms_per_step": e2e_ms,
                "note": "each rank copies its rows of X and delta (rank 0 also grad_W) from pinned host memory "
                        "every step; rank 0 reads W back"},
    }
    print(json.dumps(out), flush=True)


def run_c3(args, rank, world, local_rank):
    """8-layer MLP (1024 -> 2048, 6 x 2048 -> 2048, 2048 -> 100, ReLU), batch
    4096, x ~ N(0,1), random labels, bf16 autocast forward, use_true_bf16, factor_update_freq 10,
    momentum 0.9.  A step is forward + backward + IFKFAC.step (one refresh every 10 steps, so the
    timed steps are a multiple of 10).  The same steps are timed with the per-layer apply
    ("per_layer_apply") to show the batched solves of ifk_natgrad_batched."""
    import copy
    import torch
    from ifkfac_b200.ifkfac import IFKFAC
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(0)
    dims = [1024] + [2048] * 7 + [100]
    layers = []
    for i in range(8):
        layers.append(torch.nn.Linear(dims[i], dims[i + 1]))
        if i < 7:
            layers.append(torch.nn.ReLU())
    torch.manual_seed(0)
    base = torch.nn.Sequential(*layers).to(dev)
    x = torch.randn(4096, 1024, generator=g, device=dev)
    y = torch.randint(0, 100, (4096,), generator=g, device=dev)
    steps = max(10, (args.steps + 9) // 10 * 10)

    def timed(batched):
        model = copy.deepcopy(base)
        opt = IFKFAC(model, lr=1e-3, damping=1e-2, factor_update_freq=10, momentum=0.9, use_true_bf16=True,
                     batched_qr=args.c3_batched_qr)
        if not batched:
            opt._batched_natgrads = lambda modules: {}

        def one():
            opt.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = model(x)
            loss = torch.nn.functional.cross_entropy(out.float(), y)
            loss.backward()
            opt.step()
            return loss

        for _ in range(max(args.warmup, 10)):  # past the first refresh
            one()
        torch.cuda.synchronize()
        if args.profile:
            # a refresh step (the 20th) and a plain one, each in its own range, for a profiler
            for k in range(10):
                if k == 9:
                    torch.cuda.nvtx.range_push("ifk_profile_step")
                one()
            torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_push("ifk_profile_plain_step")
            one()
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            return 0.0, 0.0
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            loss = one()
        b.record()
        b.synchronize()
        opt.cleanup()
        return a.elapsed_time(b) / steps, float(loss.item())

    def timed_classic():
        """The control (next row f4): ClassicKFAC on the same model and steps (Gram
        matrices of the captured rows, explicit inverses every 10 steps)."""
        from ifkfac_b200.classic_kfac import ClassicKFAC
        model = copy.deepcopy(base)
        opt = ClassicKFAC(model, lr=1e-3, damping=1e-2, factor_update_freq=10, decomp_update_freq=10, momentum=0.9)

        def one():
            opt.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = model(x)
            loss = torch.nn.functional.cross_entropy(out.float(), y)
            loss.backward()
            opt.step()
            return loss

        for _ in range(max(args.warmup, 10)):
            one()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            loss = one()
        b.record()
        b.synchronize()
        opt.cleanup()
        ms = a.elapsed_time(b) / steps
        return {"ms_per_step": ms, "value": 1000.0 / ms, "final_loss": float(loss.item())}

    # the apply variants alternate (batched, per-layer, batched, per-layer) so that
    # the order of the runs in the process does not favour either; each keeps its best
    if args.profile:
        timed(not args.c3_per_layer_apply)
        return
    with ClockSampler(local_rank) as clk:
        runs = [timed(not args.c3_per_layer_apply)]
        if not args.c3_per_layer_apply:
            runs += [timed(False), timed(True), timed(False)]
        classic = timed_classic() if args.c3_classic else None
    ms, loss = min(runs[0::2]) if not args.c3_per_layer_apply else runs[0]
    ms_pl = None if args.c3_per_layer_apply else min(r[0] for r in runs[1::2])
    out = {"metric": "preconditioned steps/sec (training step: forward + backward + IFKFAC.step)",
           "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 10),
           "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic",
           "config": {"workload": "C3 8-layer MLP 1024-2048x7-100, batch 4096, bf16 autocast, use_true_bf16, "
                                  "factor_update_freq 10, momentum 0.9", "final_loss": loss,
                      "timing": "eager, CUDA events around the step loop (host work included); best of 2 runs "
                                "of each apply, alternated"},
           "batched_qr": args.c3_batched_qr, "apply": "per-layer" if args.c3_per_layer_apply else "batched",
           "per_layer_apply": {"ms_per_step": ms_pl, "value": 1000.0 / ms_pl} if ms_pl else None,
           "classic_kfac": classic,
           "clocks": clk.summary()}
    print(json.dumps(out), flush=True)


def run_c4(args, rank, world, local_rank):
    """a GPT-2-small-shaped decoder (12 blocks, d 768, 12 heads, MLP 3072,
    seq 1024, batch 8: p = 8192 tokens; vocab 50257, uniform random token ids), random init,
    bf16 autocast, K-FAC on every Linear of the blocks (qkv 768->2304, proj, fc 768->3072,
    fc2 3072->768; the 50257-wide head excluded by max_out_dim = 4096), use_true_bf16,
    damping 1e-3, every token's rows (max_seq_rows = 0), batched_qr, momentum 0.9,
    factor_update_freq 10.  A step is forward + backward + IFKFAC.step."""
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from ifkfac_b200.ifkfac import IFKFAC
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    d, heads, seq, batch, vocab = 768, 12, 1024, 8, 50257

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln1, self.ln2 = nn.LayerNorm(d), nn.LayerNorm(d)
            self.qkv, self.proj = nn.Linear(d, 3 * d), nn.Linear(d, d)
            self.fc, self.fc2 = nn.Linear(d, 4 * d), nn.Linear(4 * d, d)

        def forward(self, x):
            B, T, _ = x.shape
            q, k, v = self.qkv(self.ln1(x)).split(d, dim=2)
            q, k, v = (t.view(B, T, heads, d // heads).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            x = x + self.proj(a.transpose(1, 2).reshape(B, T, d))
            return x + self.fc2(F.gelu(self.fc(self.ln2(x))))

    class GPT(nn.Module):
        def __init__(self):
            super().__init__()
            self.tok, self.pos = nn.Embedding(vocab, d), nn.Embedding(seq, d)
            self.blocks = nn.ModuleList([Block() for _ in range(12)])
            self.ln, self.head = nn.LayerNorm(d), nn.Linear(d, vocab, bias=False)

        def forward(self, idx):
            x = self.tok(idx) + self.pos(torch.arange(idx.shape[1], device=idx.device))
            for b in self.blocks:
                x = b(x)
            return self.head(self.ln(x))

    torch.manual_seed(0)
    model = GPT().to(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    idx = torch.randint(0, vocab, (batch, seq + 1), generator=g, device=dev)
    x, y = idx[:, :-1], idx[:, 1:]
    opt = IFKFAC(model, lr=1e-3, damping=1e-3, factor_update_freq=10, momentum=0.9, use_true_bf16=True,
                 max_out_dim=4096, max_seq_rows=0, batched_qr=True)

    def one():
        opt.zero_grad()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(x)
        loss = F.cross_entropy(logits.float().reshape(-1, vocab), y.reshape(-1))
        loss.backward()
        opt.step()
        return loss

    steps = max(10, (args.steps + 9) // 10 * 10)
    for _ in range(max(args.warmup, 10)):
        one()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            loss = one()
        b.record()
        b.synchronize()
    ms = a.elapsed_time(b) / steps
    ksum = kernel_summary(one, 20) if args.kernel_summary else None
    out = {"metric": "preconditioned steps/sec (training step: forward + backward + IFKFAC.step)",
           "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 10),
           "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic", "kernel_summary": ksum,
           "config": {"workload": "C4 GPT-2-small-shaped decoder, 12 x (qkv, proj, fc, fc2) under K-FAC, "
                                  "8 x 1024 tokens, bf16 autocast, use_true_bf16, damping 1e-3, batched_qr",
                      "layers_under_kfac": len(opt.hooks.linear_layers), "final_loss": float(loss.item()),
                      "timing": "eager, CUDA events around the step loop (host work included)"},
           "clocks": clk.summary()}
    opt.cleanup()
    print(json.dumps(out), flush=True)


def kernel_summary(step_fn, steps, top=20):
    """Device time per kernel over `steps` extra calls of step_fn, under torch.profiler
    (CUPTI activity records, no kernel replay): the `top` kernels by total time, as
    ms per step and share of the kernels' total."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step_fn()
        torch.cuda.synchronize()
    rows = []
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", None)
        if t is None:
            t = e.cuda_time_total
        if t > 0:
            rows.append((t, e.key, e.count))
    rows.sort(reverse=True)
    tot = sum(r[0] for r in rows)
    return {"steps": steps, "kernels_ms_per_step": round(tot / 1e3 / steps, 2),
            "top": [{"kernel": k[:100], "ms_per_step": round(t / 1e3 / steps, 3), "share": round(t / tot, 4),
                     "launches_per_step": round(c / steps, 1)} for t, k, c in rows[:top]]}


def run_c1(args, rank, world, local_rank):
    """BASELINE config 1, the reference's CPU-runnable case: Linear(128->256)-ReLU-Linear(256->10),
    fp32, x (256, 128) ~ N(0, 1), random labels, cross-entropy, lr 1e-3, damping 1e-2,
    factor_update_freq 1 (a refresh every step), momentum 0.9, 100 steps.  Beside it, the
    same step with the curvature path in the oracle port on the host cores (forward and
    backward in torch on the CPU; QR, damping fold, solves and update in scipy LAPACK)."""
    import time
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    from ifkfac_b200.ifkfac import IFKFAC
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    base = nn.Sequential(nn.Linear(128, 256), nn.ReLU(), nn.Linear(256, 10))
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 128, generator=g)
    y = torch.randint(0, 10, (256,), generator=g)
    import copy
    model = copy.deepcopy(base).to(dev)
    xd, yd = x.to(dev), y.to(dev)
    opt = IFKFAC(model, lr=1e-3, damping=1e-2, factor_update_freq=1, momentum=0.9)

    def one():
        opt.zero_grad()
        loss = F.cross_entropy(model(xd), yd)
        loss.backward()
        opt.step()
        return loss

    for _ in range(max(args.warmup, 3)):
        one()
    torch.cuda.synchronize()
    steps = 100
    with ClockSampler(local_rank) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            loss = one()
        b.record()
        b.synchronize()
    ms = a.elapsed_time(b) / steps
    opt.cleanup()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import ifk_oracle as O
        torch.set_num_threads(os.cpu_count() or 1)
        m = copy.deepcopy(base)
        lin = [m[0], m[2]]
        caps = {}
        hs = [l.register_forward_hook(lambda mod, i, o: caps.__setitem__((mod, "x"), i[0].detach())) for l in lin]
        hs += [l.register_full_backward_hook(lambda mod, gi, go: caps.__setitem__((mod, "g"), go[0].detach()))
               for l in lin]
        bufs = {}

        def cpu_step():
            m.zero_grad()
            F.cross_entropy(m(x), y).backward()
            for l in lin:
                X, D = caps[(l, "x")].numpy(), caps[(l, "g")].numpy()
                RX = O.get_factor(O.streaming_tsqr_update(None, X), X.shape[0], 1e-2)
                RG = O.get_factor(O.streaming_tsqr_update(None, D), D.shape[0], 1e-2)
                if RX is None or RG is None:  # trapezoidal (fewer rows than columns): plain step
                    continue
                nat = O.apply_vered(l.weight.grad.numpy(), RX, RG)
                W, bufs[l] = O.precond_update(l.weight.detach().numpy(), bufs.get(l), nat, 1e-3, 0.9, 0.0, None)
                nb = O.apply_vered_bias(l.bias.grad.numpy(), RG)
                with torch.no_grad():
                    l.weight.copy_(torch.from_numpy(W))
                    l.bias.sub_(1e-3 * torch.from_numpy(nb))

        cpu_step()
        n_cpu = 20
        t0 = time.perf_counter()
        for _ in range(n_cpu):
            cpu_step()
        cpu_s = (time.perf_counter() - t0) / n_cpu
        for h in hs:
            h.remove()
        cpu = {"value": 1.0 / cpu_s, "unit": "steps/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{n_cpu} steps: torch CPU forward/backward, oracle (scipy LAPACK) curvature and update"}
    out = {"metric": "preconditioned steps/sec (training step: forward + backward + IFKFAC.step)",
           "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3),
           "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": "synthetic",
           "config": {"workload": "C1 Linear(128-256)-ReLU-Linear(256-10), batch 256, fp32, refresh every step",
                      "final_loss": float(loss.item()),
                      "timing": "eager, CUDA events around the step loop (host work included)"},
           "cpu_baseline": cpu, "clocks": clk.summary()}
    print(json.dumps(out), flush=True)


def run_c5(args, rank, world, local_rank):
    """a Llama-1B-shaped decoder (16 blocks, d 2048, 32 query and 8
    key/value heads, SwiGLU MLP 8192, vocab 128256 with the head tied to the embedding,
    RMSNorm; no rotary embedding, which does not change a K-FAC shape), random init,
    bf16 autocast, sequences of 2048 uniform random token ids.  K-FAC on the 112 Linear
    layers of the blocks (q, k, v, o, gate, up, down), use_true_bf16, damping 1e-3,
    factor_update_freq 20, batched_qr; every token's rows (max_seq_rows = 0: p = 32768
    rows per layer and step on 8 GPUs, as config 5 states), or with ``--c5-rows 2048``
    the reference's default cap of 2048 rows per layer and step (max_seq_rows None).
    A step is forward + backward + the optimizer step.

    Data-parallel over the ranks (config 5 as stated: batch 16 = 32768 tokens on 8
    GPUs, i.e. 2 sequences per GPU): each rank runs ``--c5-batch`` sequences of its
    own (weak scaling), and with more than one rank the optimizer is
    DistributedIFKFAC: the TSQR batch-sharded (each rank folds its own rows), the
    factors reduced to their layer's owner by the R-tree every 20 steps, gradients
    averaged, layers round-robined for the solves and the updated weights broadcast."""
    import torch
    import torch.distributed as dist
    import torch.nn as nn
    import torch.nn.functional as F
    from ifkfac_b200.ifkfac import IFKFAC
    from ifkfac_b200.distributed import DistributedIFKFAC
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    d, nh, nkv, ff, vocab, nblk, seq = 2048, 32, 8, 8192, 128256, 16, 2048
    batch = args.c5_batch
    hd = d // nh

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.n1, self.n2 = nn.RMSNorm(d), nn.RMSNorm(d)
            self.q, self.k, self.v = nn.Linear(d, d, bias=False), nn.Linear(d, nkv * hd, bias=False), \
                nn.Linear(d, nkv * hd, bias=False)
            self.o = nn.Linear(d, d, bias=False)
            self.gate, self.up = nn.Linear(d, ff, bias=False), nn.Linear(d, ff, bias=False)
            self.down = nn.Linear(ff, d, bias=False)

        def forward(self, x):
            B, T, _ = x.shape
            h = self.n1(x)
            q = self.q(h).view(B, T, nh, hd).transpose(1, 2)
            k = self.k(h).view(B, T, nkv, hd).transpose(1, 2)
            v = self.v(h).view(B, T, nkv, hd).transpose(1, 2)
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            x = x + self.o(a.transpose(1, 2).reshape(B, T, d))
            h = self.n2(x)
            return x + self.down(F.silu(self.gate(h)) * self.up(h))

    class Llama(nn.Module):
        def __init__(self):
            super().__init__()
            self.tok = nn.Embedding(vocab, d)
            nn.init.normal_(self.tok.weight, std=0.02)  # tied head: N(0, 1) rows would give logits ~ 45
            self.blocks = nn.ModuleList([Block() for _ in range(nblk)])
            self.norm = nn.RMSNorm(d)

        def forward(self, idx):
            x = self.tok(idx)
            for b in self.blocks:
                x = b(x)
            return F.linear(self.norm(x), self.tok.weight)  # tied head: not a K-FAC layer

    torch.manual_seed(0)  # the same initial weights on every rank
    model = Llama().to(dev)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)  # each rank its own batch shard
    idx = torch.randint(0, vocab, (batch, seq + 1), generator=g, device=dev)
    x, y = idx[:, :-1], idx[:, 1:]
    kw = dict(lr=1e-4, damping=1e-3, factor_update_freq=20, momentum=0.9, use_true_bf16=True, batched_qr=True,
              max_seq_rows=0 if args.c5_rows == "all" else None)
    opt = DistributedIFKFAC(model, **kw) if world > 1 else IFKFAC(model, **kw)

    def one():
        opt.zero_grad()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(x)
        loss = F.cross_entropy(logits.float().reshape(-1, vocab), y.reshape(-1))
        loss.backward()
        opt.step()
        return loss

    def barrier():
        if world > 1:
            dist.barrier()

    steps = max(20, (args.steps + 19) // 20 * 20)
    warm = max(args.warmup, 20)
    for _ in range(warm):  # past the first refresh
        one()
    torch.cuda.synchronize()
    barrier()
    with ClockSampler(local_rank) as clk:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            loss = one()
        b.record()
        b.synchronize()
    barrier()
    ms = a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ksum = kernel_summary(one, 20) if args.kernel_summary and world == 1 else None
    peak = torch.cuda.max_memory_allocated(dev) / 1e9
    if rank == 0:
        tokens = world * batch * seq
        out = {"metric": "training tokens/s (forward + backward + IFKFAC.step, K-FAC on 112 layers)",
               "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
               "warmup": warm, "ms_per_step": ms, "steps_per_s": 1000.0 / ms, "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
               "config": {"workload": "C5 Llama-1B-shaped decoder, 16 x (q, k, v, o, gate, up, down) under "
                                      "K-FAC, " + ("every token's rows" if args.c5_rows == "all" else
                                                   "2048 rows per layer, rank and step") +
                                      ", bf16 autocast, use_true_bf16, damping 1e-3, factor_update_freq 20, batched_qr",
                          "rows_per_layer_per_step": (world * batch * seq if args.c5_rows == "all" else world * 2048),
                          "sequences_per_gpu": batch, "seq_len": seq, "global_batch": world * batch,
                          "parallelism": ("single GPU" if world == 1 else
                                          f"data parallel over {world} GPUs: TSQR batch-sharded, R-tree to the "
                                          "layer owners every 20 steps, layers round-robined for the solves"),
                          "layers_under_kfac": len(opt.hooks.linear_layers), "final_loss": float(loss.item()),
                          "timing": "eager, CUDA events around the step loop (host work included), max over ranks"},
               "peak_mem_gb": peak, "clocks": clk.summary(), "kernel_summary": ksum}
        print(json.dumps(out), flush=True)
    opt.cleanup()


def run_laplace(args, rank, world, local_rank):
    """Next-row f4, the K-FAC Laplace posterior (ifkfac/laplace.py) of one 4096 x 4096
    layer, N = 50000, prior precision 1e-2.  Square roots R_A, R_G come from folding
    16384 bf16 rows each.  Ours: the precision factors C (ifk_finalize, two in one call
    each) and draws C_G^-1 xi C_A^-T (ifk_posterior_sample), bf16 mode.  Beside it, on
    the same GPU, the reference's route: svd(R) of both factors (torch/cuSOLVER) and
    the draw U_G diag xi diag U_A^T (two fp32 GEMMs); and the oracle on host cores."""
    import time
    import torch
    from ifkfac_b200 import _lib
    from ifkfac_b200.engine import Factor, fold_segments
    from ifkfac_b200.laplace import posterior_factors, posterior_sample
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    n, p, N, lam = N_DIM, 16384, 50000, 1e-2
    g = torch.Generator(device=dev).manual_seed(0)
    Rs = []
    for _ in range(2):
        s = torch.exp(torch.rand(n, generator=g, device=dev) * math.log(100.0))
        f = Factor(n, dev, _lib.PREC_BF16)
        fold_segments((f,), ([(torch.randn(p, n, generator=g, device=dev) * s).bfloat16()],), None)
        Rs.append((f.R / math.sqrt(p)).contiguous())
    torch.cuda.synchronize()
    xi = torch.randn(n, n, generator=g, device=dev)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            out = fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps, out

    with ClockSampler(local_rank) as clk:
        t_fac, C = timed(lambda: posterior_factors(Rs, N, lam, torch.bfloat16, _lib.PREC_BF16), 5)
        t_draw, dW = timed(lambda: posterior_sample(xi, C[0], C[1], _lib.PREC_BF16), max(args.steps, 10))
        C32 = posterior_factors(Rs, N, lam, torch.float32, _lib.PREC_FP32)
        t_draw32, _ = timed(lambda: posterior_sample(xi, C32[0], C32[1], _lib.PREC_FP32), 5)
        t_svd, evd = timed(lambda: [torch.linalg.svd(R) for R in Rs], 1)
        U_A, U_G = evd[0][2].T.contiguous(), evd[1][2].T.contiguous()
        sA = 1.0 / torch.sqrt(math.sqrt(N) * evd[0][1] ** 2 + math.sqrt(lam))
        sG = 1.0 / torch.sqrt(math.sqrt(N) * evd[1][1] ** 2 + math.sqrt(lam))
        t_evd, _ = timed(lambda: U_G @ (xi * sG[:, None] * sA[None, :]) @ U_A.T, max(args.steps, 10))
    assert torch.isfinite(dW).all()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import ifk_oracle as O
        RA, RG = (R.double().cpu().numpy() for R in Rs)
        t0 = time.perf_counter()
        CA, CG = O.posterior_factor(RA, N, lam), O.posterior_factor(RG, N, lam)
        t1 = time.perf_counter()
        O.posterior_sample(CA, CG, xi.double().cpu().numpy())
        t2 = time.perf_counter()
        cpu = {"value": 1.0 / (t2 - t1), "unit": "draws/s", "cores": os.cpu_count(), "kind": "port",
               "sample": "one fp64 factor pair build (%.2f s) and one draw on the host" % (t1 - t0)}
    out = {"metric": "K-FAC Laplace posterior draws/s (one 4096 x 4096 layer)", "value": 1000.0 / t_draw,
           "unit": "draws/s", "n_gpus": 1, "ms_per_draw": t_draw, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "f4 Laplace: C = qr([N^1/4 R; lambda^1/4 I]) per side, draw C_G^-1 xi C_A^-T",
                      "N": N, "prior_precision": lam},
           "factor_build_ms": t_fac, "draw_fp32_mode_ms": t_draw32,
           "reference_route_gpu": {"svd_of_both_factors_ms": t_svd, "evd_draw_ms": t_evd},
           "cpu_baseline": cpu, "clocks": clk.summary()}
    print(json.dumps(out), flush=True)


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class RefOperator:
    """The reference's executed config-2 path on the host cores, cut into eight slices.

    Slice s (s = 0 .. 7) folds row tile s of X and of delta into the running factors
    with ``streaming_tsqr_update`` (``ifkfac/triangular.py:246-307``: leaf QR and merge
    QR, both ``torch.linalg.qr(mode="reduced")``, which also forms Q); slice 7 then
    finalises both factors (``get_factors`` / ``finalize_R``,
    ``ifkfac/activation_hooks.py:323-332``, ``ifkfac/triangular.py:386-421``), casts
    them to bf16 (``ifkfac/ifkfac.py:292-294``), runs the four fp32 solves of the
    bf16-stored dispatch (``ifkfac/triangular.py:607-628``) and the momentum / lr
    update (``ifkfac/ifkfac.py:394-413``).  Eight consecutive slices are one whole
    operator; nothing is extrapolated.  The calls are those of the reference, on
    torch's CPU LAPACK (``oracle/torch_port.py``), fed the fp32 upcast of the bf16
    rows (the reference's QR has no bf16 kernel)."""

    NSLICE = P_ROWS // TILE

    def __init__(self, seed=0):
        import torch
        from oracle import torch_port as TP
        self.TP = TP
        g = torch.Generator().manual_seed(seed)

        def scaled():
            s = torch.exp(torch.rand(N_DIM, generator=g) * math.log(100.0))
            return (torch.randn(P_ROWS, N_DIM, generator=g) * s).to(torch.bfloat16).float()

        self.X, self.D = scaled(), scaled()
        self.gW = torch.randn(N_DIM, N_DIM, generator=g) * 1e-2
        self.W = torch.randn(N_DIM, N_DIM, generator=g) * 1e-2
        self.buf = None
        self.RX = self.RG = None

    def slice(self, s):
        import torch
        TP = self.TP
        lo, hi = s * TILE, (s + 1) * TILE
        if s == 0:
            self.RX = self.RG = None
        self.RX = TP.streaming_tsqr_update(self.RX, self.X[lo:hi])
        self.RG = TP.streaming_tsqr_update(self.RG, self.D[lo:hi])
        if s == self.NSLICE - 1:
            fx = TP.get_factor(self.RX, P_ROWS, DAMPING).to(torch.bfloat16)
            fg = TP.get_factor(self.RG, P_ROWS, DAMPING).to(torch.bfloat16)
            nat = TP.apply_vered_bf16_stored(self.gW, fx, fg)
            self.buf = TP.precond_update_(self.W, self.buf, nat, LR, MOM)


def _slice_times(op, first, count):
    """Run `count` slices starting at slice index `first`; returns [(slice, seconds)]."""
    out = []
    for i in range(first, first + count):
        s = i % op.NSLICE
        t0 = time.perf_counter()
        op.slice(s)
        out.append((s, time.perf_counter() - t0))
    return out


def _operator_seconds(samples):
    """Seconds of one whole operator: the sum over the eight slices of each slice's
    mean measured time."""
    by = {}
    for s, t in samples:
        by.setdefault(s, []).append(t)
    return sum(sum(v) / len(v) for v in by.values()), sorted(by)


def cpu_baseline():
    """The reference's executed path on the host cores: one whole config-2 operator
    (eight slices of RefOperator), timed once, all host threads."""
    import torch
    torch.set_num_threads(os.cpu_count())
    op = RefOperator(0)
    samples = _slice_times(op, 0, op.NSLICE)
    sec, _ = _operator_seconds(samples)
    return {"value": 1.0 / sec, "unit": "steps/s", "cores": torch.get_num_threads(), "kind": "port",
            "cpu_model": _cpu_model(),
            "sample": ("one whole config-2 operator on the host cores: the reference's calls "
                       "(torch.linalg.qr mode='reduced' leaf + merge per 2048-row tile of X and delta, "
                       "finalize_R, bf16 cast, four fp32 solve_triangular, momentum update) on torch's CPU "
                       f"LAPACK, fp32 upcast of the bf16 rows; {sec:.1f} s measured, not extrapolated"),
            "sample_seconds": sec}


def run_reference(args, rank, world):
    """Reference arm: the reference's CPU path (its own torch.linalg calls, restated in
    oracle/torch_port.py, since the reference is Python and does not travel to the GPU
    box) on all host cores; rank 0 only.  Each step is one slice of the operator (one
    row tile of X and delta folded; the last slice of eight also finalises, solves and
    updates), so eight consecutive steps are one whole operator.  The value is whole
    operators per second: 1 / (sum over the eight slices of their mean time in the timed
    steps); ms_per_step is the measured time of a timed step."""
    if rank != 0:
        return
    import torch
    torch.set_num_threads(os.cpu_count())
    op = RefOperator(0)
    warm = _slice_times(op, 0, args.warmup)
    t0 = time.perf_counter()
    timed = _slice_times(op, args.warmup, args.steps)
    wall = time.perf_counter() - t0
    seen = {s for s, _ in timed}
    extra = []
    if len(seen) < op.NSLICE:  # fewer than 8 timed steps: complete the cycle outside the timed region
        extra = [x for x in warm if x[0] not in seen]
        seen |= {s for s, _ in extra}
        missing = [s for s in range(op.NSLICE) if s not in seen]
        if missing:
            extra += _slice_times(op, missing[0], op.NSLICE - missing[0])
    sec, _ = _operator_seconds(timed + [x for x in extra if x[0] not in {s for s, _ in timed}])
    v = 1.0 / sec
    ms = 1000.0 * wall / max(args.steps, 1)
    cb = {"value": v, "unit": "steps/s", "cores": torch.get_num_threads(), "kind": "port",
          "cpu_model": _cpu_model(),
          "sample": ("each step one eighth of the config-2 operator (one 2048-row tile of X and delta folded "
                     "with the reference's torch.linalg.qr mode='reduced' leaf + merge; the eighth slice also "
                     "finalize_R, bf16 cast, four fp32 solves, momentum update); operator time = sum over "
                     f"the eight slices of their mean measured time = {sec:.2f} s")}
    out = {"impl": "reference", "metric": METRIC, "value": v, "unit": "steps/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "operator_seconds": sec,
           "config": {"workload": WORKLOAD, "n": N_DIM, "p": P_ROWS, "tile_rows": TILE,
                      "damping": DAMPING, "lr": LR, "momentum": MOM, "use_true_bf16": True},
           "cpu_baseline": cb,
           "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5", "laplace"], default="c2",
                    help="c1: the reference's CPU-runnable MLP; c2: the single-layer operator (the headline); "
                         "c3: the 8-layer MLP training step; "
                         "c4: the GPT-2-small-shaped decoder training step; c5: the Llama-1B-shaped one, data parallel "
                         "over the ranks; "
                         "laplace: K-FAC Laplace draws")
    ap.add_argument("--c5-batch", type=int, default=2,
                    help="c5: sequences of 2048 tokens per GPU (config 5: 16 on 8 GPUs, i.e. 2 per GPU)")
    ap.add_argument("--c5-rows", choices=["all", "2048"], default="all",
                    help="c5: fold every token's rows (config 5: p = 32768 on 8 GPUs) or the reference's "
                         "default cap of 2048 rows per layer and step")
    ap.add_argument("--c3-batched-qr", action="store_true",
                    help="c3: IFKFAC(batched_qr=True): the step's chunks of every layer folded together")
    ap.add_argument("--c3-per-layer-apply", action="store_true", help="c3: time only the per-layer apply")
    ap.add_argument("--kernel-summary", action="store_true",
                    help="c4, c5: after the timed steps, profile 20 more (torch.profiler) and add the top kernels")
    ap.add_argument("--c3-classic", action="store_true",
                    help="c3: also time the ClassicKFAC comparator on the same model and steps")
    ap.add_argument("--schedule", choices=["one-launch", "per-tile"], default="one-launch",
                    help="fold schedule of the timed step (the other one is reported beside it)")
    ap.add_argument("--e2e-groups", default="1",
                    help="one-launch schedule, e2e: fold launches the row tiles are split into: a count of "
                         "equal groups, or comma-separated tile counts of consecutive groups (e.g. 1,7)")
    ap.add_argument("--partition", choices=["rows", "layers"], default="rows",
                    help="N > 1, config 2: 'rows' (default) solves the same operator on N GPUs, rows "
                         "batch-sharded and merged by the R-tree; 'layers' gives every rank a layer of its own "
                         "(independent operators, no collective)")
    ap.add_argument("--no-fp32-mode", action="store_true",
                    help="skip the secondary timing of the fp32 mode (use_true_bf16=False)")
    ap.add_argument("--no-other-schedule", action="store_true",
                    help="skip the secondary timing of the other schedule")
    ap.add_argument("--profile", action="store_true",
                    help="run --warmup eager steps and one more step, then exit (for ncu)")
    ap.add_argument("--profile-size", choices=["full", "small"], default="full",
                    help="with --profile: 'small' runs n=1024, p=4096, tiles of 1024 (short ncu captures)")
    args = ap.parse_args()
    if args.profile and args.profile_size == "small":
        global N_DIM, P_ROWS, TILE
        N_DIM, P_ROWS, TILE = 1024, 4096, 1024
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)  # rank 0 only; other ranks exit without work
        return
    if args.config in ("c1", "c3", "c4", "laplace"):
        if rank == 0:
            runs = {"c1": run_c1, "c3": run_c3, "c4": run_c4, "laplace": run_laplace}
            runs[args.config](args, rank, world, local_rank)
        return
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local_rank))
    try:
        if args.config == "c5":
            run_c5(args, rank, world, local_rank)
        elif world > 1 and args.partition == "rows":
            run_sharded(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
