#!/usr/bin/env python
"""Headline benchmark: forward + backward solves of the large single-family problem.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--config 3]
    python bench.py --config 4 [--families F --chunk F_c]       # the batched-family workload
    python bench.py --config 5 [--directions D]                 # forward + D-direction tangent

One "step" is one full solve on every GPU: ``run_forward`` (E fixed point, every wave's split
reduction and pi_iters sweeps, NLL) + ``run_backward`` (implicit adjoint, E-adjoint BiCGSTAB,
theta VJP) on the benchmark's config-3 family (S=4095 columns, ~131k rows, pi_iters=16,
neumann_terms=16, seeded synthetic data).  With N GPUs (torchrun, one process per GPU) each rank
solves its own family (seed 3000+rank) and the packed [loss, grad_theta, grad_col] is summed with
one NCCL all-reduce per step -- the family-sharded data-parallel step; per-GPU work is fixed
("weak" scaling).  ``value`` is the whole-job solves/s timed on the device (max over ranks);
``e2e`` is the same step through the public API with theta/col_weights copied from pinned host
memory and the loss + gradients copied back every step.

``--impl reference`` times the reference's own implementation on the host cores: its runtime and
kernels under the Triton interpreter, on a bounded sample of the same workload (a family with the
same species tree and fewer rows), extrapolated per row (the line states the formula), one
single-threaded process per host thread, all started together; the numpy port of the same
algorithm (``oracle/``) is reported beside it.  On N>1 only rank 0 runs it.

``--atomic-backward`` runs the headline backward with atomic child adds instead of its default
deterministic form (child adjoints gathered from edge rows in a fixed order).

``--config 4`` measures the batched workload instead: 1024 families (S=1023, ~16k rows each)
sharing one theta, split into contiguous blocks per rank, each block processed in chunks of
``--chunk`` families (all 1024 families' [C,S] state, ~275 GB, does not fit one GPU), with one
all-reduce of [loss, column accumulators] per step; ``value`` is families/s.

``--config 5`` measures the tangent workload: the config-3 family's forward plus the forward-mode
tangent of the root scores along 32 directions (one batched pass), checked against central
finite differences of the forward; ``value`` is tangent passes/s (forward + all directions).
"""

from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "kernel-bench_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "fwd+bwd solves/sec (S=4095, C~131k single family per GPU; BASELINE config 3)"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the strong-scaled batched workload (config 4) measured beside the headline")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's own Triton path on this GPU (baseline/_ref) at N=1")
    ap.add_argument("--families", type=int, default=None, help="config 4: families in the whole batch")
    ap.add_argument("--chunk", type=int, default=128, help="config 4: families per chunk on a GPU")
    ap.add_argument("--host-builder", action="store_true",
                    help="config 4: build the static layouts and schedules on the host instead of the device")
    ap.add_argument("--directions", type=int, default=32, help="config 5: tangent directions per pass")
    ap.add_argument("--hvp", action="store_true",
                    help="exact-Hessian HVPs/s (newton/hvp_exact.py) on the --hvp-config family")
    ap.add_argument("--hvp-config", type=int, default=2, help="--hvp: the problem config (default 2, S=511)")
    ap.add_argument("--traffic-case", nargs="?", const="reduced", choices=("reduced", "config3"), default=None,
                    help="two forward + backward passes and nothing else, for ncu captures: 'reduced' (default) is "
                         "a reduced config-3 family (the config-3 species tree, 2,048 genes: ~12.7k rows, 208 MB per "
                         "[C,S] buffer) for multi-pass captures; 'config3' is the full config-3 family, for "
                         "single-pass captures (DRAM bytes, durations) of the full-size launches")
    ap.add_argument("--per-kernel", action="store_true",
                    help="per-wrapper times of one forward + backward pass driven by the reference's own glue, "
                         "over the reference's stock Triton kernels and over this project's (--config, default 2)")
    ap.add_argument("--atomic-backward", action="store_true",
                    help="run the headline backward with atomic child adds instead of its deterministic form "
                         "(child adjoints gathered from edge rows in a fixed order; engine._edge_scratch)")
    ap.add_argument("--cuda-profiler-range", action="store_true",
                    help="bracket the timed region with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    return ap.parse_args()


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.tmp, stderr=subprocess.DEVNULL)
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
        self.tmp.flush()
        text = Path(self.tmp.name).read_text()
        os.unlink(self.tmp.name)
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for row in csv.reader(io.StringIO(text)):
            if len(row) < 9:
                continue
            try:
                sm.append(float(row[1]))
                smax = float(row[2])
            except ValueError:
                continue
            for n, v in zip(names, row[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def algorithmic_bytes(plan, S):
    """Compulsory-touch bytes per level: forward writes Pi and Pibar of every row and reads Pi and
    Pibar of each distinct child row the level references once; backward reads Pi, Pibar and the
    adjoint of every row, re-reads each distinct child's Pi and Pibar and read-modify-writes its
    adjoint row (fp32)."""
    fwd, bwd = {}, {}
    for L in range(plan.n_levels):
        n = plan.level_ptr[L + 1] - plan.level_ptr[L]
        k = plan.children_per_level[L]
        fwd[L] = 4 * S * (2 * n + 2 * k)
        bwd[L] = 4 * S * (3 * n + 4 * k)
    return fwd, bwd


# Counters of ONE launch of each dataflow kernel on the benchmark's own config-3 family (seed 3000,
# C = 128,282 rows), from single-pass ncu captures of the full-size launches
# (``bench.py --traffic-case config3``): DRAM bytes read and written, and warp instructions
# executed; the backward's per form (its child adjoints gathered from edge rows, the default, or
# added with atomics).  A form not captured for the current build reports null.
CONFIG3_ROWS = 128282
CONFIG3_COUNTERS: dict = {
    "kb_flow_forward": {"dram_read": 18417902080, "dram_write": 6217162240, "warp_inst": 23781305587},
    ("kb_flow_backward", "atomic"): {"dram_read": 45366837504, "dram_write": 16917131776,
                                     "warp_inst": 40822535893},
    ("kb_flow_backward", "deterministic"): {"dram_read": 85957630464, "dram_write": 42019007232,
                                            "warp_inst": 43715164395},
}


def launch_counters(name, C, S, form=None):
    """The captured counters of one launch of ``name`` (the backward: in ``form``) on the config-3
    family, else None."""
    if S != 4095 or C != CONFIG3_ROWS:
        return None
    return CONFIG3_COUNTERS.get(name if form is None else (name, form))


def issue_roofline(warp_inst, ms, sm_mhz):
    """Issue-slot bound of a launch: 148 SMs x 4 schedulers x one warp instruction per clock at
    the sampled SM clock; ``frac`` = that minimum time / the measured time."""
    min_ms = warp_inst / (148 * 4 * float(sm_mhz) * 1e6) * 1e3
    return {"warp_inst_per_launch": int(warp_inst), "min_ms": round(min_ms, 3), "sm_mhz": float(sm_mhz),
            "frac": round(min_ms / ms, 4)}


def kernel_bytes(name, per, fwd_b, bwd_b):
    """Algorithmic bytes of the launches ``per`` [(level, ms)] of one engine kernel: a level launch
    covers its level, a dataflow launch (kb_flow_*) the whole sweep."""
    bm = fwd_b if "forward" in name else bwd_b
    if name.startswith("kb_flow_"):
        return len(per) * sum(bm.values())
    return sum(bm[lv] for lv, _ in per)


def cpu_sample_case(n_genes, S_species_leaves=2048):
    """A bounded sample of the workload for the CPU oracle: the benchmark's species tree size
    with a small gene family (same per-row work, fewer rows)."""
    from kbench_b200 import gen
    return gen.ProblemConfig("cpu_sample", S_species_leaves, n_genes, 2, max(8, n_genes // 3), 0,
                             solver_options=dict(gen.CONFIGS[3].solver_options))


def run_cpu_oracle_sample(full_rows, seed, n_genes=512, species_leaves=2048):
    """Time the oracle (forward + backward) on the sample; returns (solves/s, seconds, rows)."""
    run, rows = _oracle_sample_fn("solve", (n_genes, species_leaves, seed))
    t0 = time.perf_counter()
    run()
    dt = time.perf_counter() - t0
    # per-row work is the same (same S, same iteration counts): scale to the full family
    solve_s = dt * full_rows / rows
    return 1.0 / solve_s, dt, rows


def host_threads():
    """Host threads this process may run on (its CPU affinity), capped at 64 sample processes."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, 64))


def _oracle_sample_fn(kind, params):
    """Builds a bounded oracle sample (untimed); returns (run, rows): run() performs one timed pass
    -- forward + backward for kind "solve" (params: n_genes, species leaves, seed), one HVP with the
    point cache prebuilt for kind "hvp" (params: config, seed, n_genes)."""
    import numpy as np
    from kbench_b200 import gen
    from oracle import kb_oracle as O
    if kind == "solve":
        n_genes, leaves, seed = params
        cap = gen.generate(cpu_sample_case(n_genes, leaves), seed=seed, as_torch=False)
    else:
        cfg, seed, n_genes = params
        c = gen.CONFIGS[cfg]
        case = gen.ProblemConfig("hvp_sample", c.n_species, n_genes, 2, max(4, n_genes // 3), 0,
                                 solver_options=dict(c.solver_options))
        cap = gen.generate(case, seed=seed, as_torch=False)
    st = dict(cap["static"])
    st["solver_options"] = cap["meta"]["solver_options"]
    theta, cw = cap["inputs"]["theta"], cap["inputs"]["col_weights"]
    rows = int(cap["meta"]["C"])
    if kind == "solve":
        def run():
            _, saved = O.forward(st, theta, cw)
            O.backward(st, theta, cw, saved)
        return run, rows
    from oracle import kb_oracle_hvp as OH
    _, saved = O.forward(st, theta, cw)
    cache = OH.point_cache(st, theta, cw, saved)
    u = np.random.default_rng(seed).standard_normal(theta.size).astype(np.float32)
    return (lambda: OH.hvp(st, theta, cw, saved, u, cache=cache)), rows


def _oracle_worker(kind, params, n_iter, barrier, out_q, idx):
    """One single-threaded sample process of parallel_oracle (module level: spawn imports it)."""
    try:
        run, rows = _oracle_sample_fn(kind, params)
        dts = []
        for _ in range(n_iter):
            barrier.wait(1800)  # every process starts its pass together
            t0 = time.perf_counter()
            run()
            dts.append(time.perf_counter() - t0)
        out_q.put((idx, rows, dts, None))
    except BaseException as exc:  # reported to the parent, which raises
        barrier.abort()
        out_q.put((idx, 0, [], repr(exc)))


def parallel_oracle(kind, params, n_iter, n_proc):
    """Runs the same bounded oracle sample in n_proc spawned single-threaded processes at once,
    n_iter passes each, every pass started together behind a barrier; returns (rows of one sample,
    per-pass wall time = the slowest process's).  Throughput of the host = n_proc samples per
    wall time."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    saved_env = {k: os.environ.get(k) for k in keys}
    for k in keys:
        os.environ[k] = "1"
    try:
        barrier = ctx.Barrier(n_proc)
        q = ctx.Queue()
        procs = [ctx.Process(target=_oracle_worker, args=(kind, params, n_iter, barrier, q, i), daemon=True)
                 for i in range(n_proc)]
        for p in procs:
            p.start()
        import queue as _queue
        results = []
        while len(results) < n_proc:
            try:
                results.append(q.get(timeout=5))
            except _queue.Empty:
                dead = [p for p in procs if p.exitcode not in (None, 0)]
                if dead:  # a process died without reporting (killed, out of memory)
                    for p in procs:
                        if p.is_alive():
                            p.terminate()
                    raise RuntimeError(f"oracle sample process exited with code {dead[0].exitcode}")
        for p in procs:
            p.join(60)
    finally:
        for k, v in saved_env.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    errors = [r[3] for r in results if r[3]]
    if errors:
        raise RuntimeError(f"oracle sample process failed: {errors[0]}")
    rows = results[0][1]
    walls = [max(r[2][i] for r in results) for i in range(n_iter)]
    return rows, walls


HVP_BYTES_PER_ROW_ELEM = 13 * 4


def traffic_case(args):
    """--traffic-case: two forward + backward passes, nothing timed, for ncu.  'reduced': a
    config-3 species tree with a smaller gene family, small enough for multi-pass captures (the
    full set of sections); 'config3': the benchmark's family itself, for single-pass metrics
    (DRAM bytes read / written and durations) of the full-size launches."""
    import torch
    from kbench_b200 import engine, gen, runtime
    if args.traffic_case == "config3":
        cfg = 3
    else:
        cfg = gen.ProblemConfig("traffic", gen.CONFIGS[3].n_species, 2048, 32, 682, 0,
                                solver_options=dict(gen.CONFIGS[3].solver_options))
    cap = gen.generate(cfg, seed=3000)
    static = runtime.make_static(cap, "cuda")
    theta, cw = cap["inputs"]["theta"].cuda(), cap["inputs"]["col_weights"].cuda()
    engine.build_plan(static)
    for _ in range(2):
        loss, saved = runtime.run_forward(static, theta, cw)
        runtime.run_backward(static, theta, cw, saved)
    torch.cuda.synchronize()
    print(json.dumps({"traffic_case": True, "C": int(cap["meta"]["C"]), "S": int(cap["meta"]["S"]),
                      "loss": float(loss)}), flush=True)


def hvp_oracle_sample(cfg, seed, n_genes):
    """Time one oracle HVP (point cache excluded) on a small family of config ``cfg``'s species
    tree; returns (seconds per HVP, rows of the sample)."""
    run, rows = _oracle_sample_fn("hvp", (cfg, seed, n_genes))
    t0 = time.perf_counter()
    run()
    return time.perf_counter() - t0, rows


def hvp_arm(args, world, rank, local):
    """--hvp: analytic exact-Hessian HVPs (forward over reverse) at a fixed point of the
    --hvp-config family, as a Newton-CG inner loop runs them (point cache built once, untimed);
    replicas on N>1."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from kbench_b200 import _lib, gen, hvp, runtime

    cfg = int(args.hvp_config)
    dev = torch.device("cuda", local if world > 1 else 0)
    cap = gen.generate(cfg, seed=1000 * cfg + rank)
    S, C = int(cap["meta"]["S"]), int(cap["meta"]["C"])
    static = runtime.make_static(cap, dev)
    theta = cap["inputs"]["theta"].to(dev)
    cw = cap["inputs"]["col_weights"].to(dev)
    _, sv = runtime.run_forward(static, theta, cw)
    torch.cuda.synchronize()
    c0 = time.perf_counter()
    f = hvp.make_exact_hvp(static, theta, cw, sv, graph=True)
    f(torch.zeros((3 * S,), device=dev))  # capture the CUDA graph (part of the one-off setup)
    torch.cuda.synchronize()
    cache_ms = (time.perf_counter() - c0) * 1e3
    U = torch.from_numpy(np.random.default_rng(7).standard_normal((4, 3 * S)).astype(np.float32)).to(dev)
    for i in range(args.warmup):
        f(U[i % 4])
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = sum(_lib.LAUNCHES.values())
    if sampler:
        sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.cuda_profiler_range:
        torch.cuda.profiler.start()
    e0.record()
    for i in range(args.steps):
        f(U[i % 4])
    e1.record()
    torch.cuda.synchronize()
    if args.cuda_profiler_range:
        torch.cuda.profiler.stop()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    launches = sum(_lib.LAUNCHES.values()) - launches0
    ms_t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    # symmetry of the operator (u1 . H u0 = u0 . H u1 up to the solves' truncation)
    h0, h1 = f(U[0]).double(), f(U[1]).double()
    asym = abs(float(U[1].double() @ h0) - float(U[0].double() @ h1)) / float(
        h0.norm() * U[1].double().norm() + h1.norm() * U[0].double().norm())
    # end to end: the direction from pinned host memory, H u back
    u_host = U.cpu().pin_memory()
    out_host = torch.empty((3 * S,), dtype=torch.float32).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for i in range(args.steps):
        out_host.copy_(f(u_host[i % 4].to(dev, non_blocking=True)), non_blocking=True)
        torch.cuda.current_stream().synchronize()
        float(out_host[0])
    x1.record()
    torch.cuda.synchronize()
    x_t = torch.tensor([x0.elapsed_time(x1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(x_t, op=dist.ReduceOp.MAX)
    e_ms = float(x_t.item())
    if rank == 0:
        peak, peak_kind = measured_peak()
        alg = HVP_BYTES_PER_ROW_ELEM * C * S
        achieved = alg / (ms * 1e-3) / 1e9
        cpu = None
        if not args.no_cpu_baseline:
            dt, rows = hvp_oracle_sample(cfg, seed=77, n_genes=24)
            per = dt * C / rows
            cpu = {"value": round(1.0 / per, 6), "unit": "HVPs/s", "cores": 1, "kind": "port",
                   "sample": f"numpy oracle HVP of a {rows}-row family on the config-{cfg} species tree (S={S}), "
                             f"{dt:.1f} s, extrapolated per row to C={C}"}
        line = {
            "metric": f"exact-Hessian HVPs/sec (newton/hvp_exact.py, config {cfg}: S={S}, C={C})",
            "value": round(world * 1000.0 / ms, 4), "unit": "HVPs/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator of the benchmark's config text)",
            "config": {"workload": f"config{cfg} HVP at a fixed point: tangent forward + tangent-adjoint sweep over "
                                   f"{int(cap['meta']['n_waves'])} waves + E side + head, replayed from one CUDA "
                                   f"graph; point cache + capture {cache_ms:.0f} ms once, untimed",
                       "parallelism": f"dp{world} (replicas)",
                       "l2": "state arrays re-read every HVP; no flush"},
            "point_cache_ms": round(cache_ms, 1), "symmetry_rel": asym,
            "roofline": {"bound": "hbm", "kernel": "whole HVP (graph of per-wave launches)", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 5),
                         "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                         "algorithmic_bytes_per_launch": alg},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * 1000.0 / e_ms, 4), "unit": "HVPs/s", "h2d_bytes_per_step": 3 * S * 4,
                    "d2h_bytes_per_step": 3 * S * 4},
            "gpu_launches": int(launches), "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def reference_hvp_arm(args, world):
    """--impl reference --hvp: the oracle port of ``newton/hvp_exact.py`` on the host cores (one
    HVP per step on a bounded sample of the --hvp-config family, extrapolated per row)."""
    from kbench_b200 import gen
    cfg = int(args.hvp_config)
    full = gen.generate(cfg, as_torch=False)["meta"]
    C, S = int(full["C"]), int(full["S"])
    n_proc = host_threads()
    rows, walls = parallel_oracle("hvp", (cfg, 77, 24), args.warmup + args.steps, n_proc)
    # n_proc HVP samples per wall time; a full HVP is C / rows samples
    step_s = statistics.median(walls[args.warmup:]) * C / rows / n_proc
    value = 1.0 / step_s
    sample = (f"numpy oracle HVP of a {rows}-row family on the config-{cfg} species tree (S={S}), "
              f"{n_proc} single-threaded processes at once, extrapolated per row to C={C}")
    print(json.dumps({
        "metric": f"exact-Hessian HVPs/sec (newton/hvp_exact.py, config {cfg}: S={S}, C={C})", "value": value,
        "unit": "HVPs/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded generator)", "impl": "reference",
        "config": {"workload": f"config{cfg} HVP, CPU sample", "sample_rows": rows},
        "cpu_baseline": {"value": value, "unit": "HVPs/s", "cores": n_proc, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "HVPs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def reference_interpreter_sample(full_rows, n_proc, genes=8):
    """The reference's own code on the host cores (``baseline/interpreter.py``: its stock runtime
    and Triton kernels under ``TRITON_INTERPRET=1``): ``n_proc`` processes started together, each
    one forward + backward of a ``genes``-gene family on the config-3 species tree.  Returns the
    per-process results and the solve time of a ``full_rows``-row family extrapolated per row."""
    from baseline import interpreter
    why = interpreter.unavailable_reason()
    if why:
        return None, why
    runs = interpreter.parallel(("sample", genes, 3000), n_proc)
    rows = runs[0]["rows"]
    med = statistics.median(r["solve_s"] for r in runs)
    return {"runs": n_proc, "sample_rows": rows, "sample_solve_s_median": round(med, 2),
            "solve_s_extrapolated": med * full_rows / rows / n_proc}, None


def reference_arm(args, world, rank):
    """--impl reference: the reference's own implementation on the host cores (its runtime and
    Triton kernels under the Triton interpreter, on a bounded sample, extrapolated per row), with
    the numpy port of the same algorithm as a secondary figure."""
    if rank != 0:
        return
    if args.hvp:
        reference_hvp_arm(args, world)
        return
    from kbench_b200 import gen
    batched = args.config == 4
    if batched:
        n_total = int(args.families or gen.CONFIGS[4].n_families)
        full_rows = int(gen.generate(4, n_families=1, as_torch=False)["meta"]["C"])  # one family
        leaves = gen.CONFIGS[4].n_species
    else:
        full_rows = int(gen.generate(args.config, as_torch=False)["meta"]["C"])
        leaves = gen.CONFIGS[3].n_species
    n_proc = host_threads()
    S = 2 * leaves - 1

    def per_step(solve_s):
        if batched:
            return solve_s * n_total, n_total / (solve_s * n_total)
        return solve_s, 1.0 / solve_s

    if batched:
        unit, metric = "families/s", "fwd+bwd families/sec (batched config 4: S=1023, ~16k rows per family, shared theta)"
        what = f"extrapolated per row to one {full_rows}-row family, x{n_total} families"
    else:
        unit, metric = "solves/s", METRIC
        what = f"extrapolated per row to C={full_rows}"
    # secondary: the numpy port of the same algorithm, W + K passes
    rows_p, walls = parallel_oracle("solve", (48, leaves, 3000), args.warmup + args.steps, n_proc)
    port_step_s, port_value = per_step(statistics.median(walls[args.warmup:]) * full_rows / rows_p / n_proc)
    port = {"value": port_value, "unit": unit, "cores": n_proc, "kind": "port", "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": port_step_s * 1e3,
            "sample": f"numpy oracle forward+backward of a {rows_p}-row family on the config-{args.config} species "
                      f"tree (S={S}), {n_proc} single-threaded processes at once, {what}"}
    # primary: the reference's own runtime and kernels under the Triton interpreter (one pass; a
    # pass is ~30 s of CPU per process, so the requested K / W apply to the port only)
    interp, why = reference_interpreter_sample(full_rows, n_proc)
    if interp is None:
        value, step_s, kind, cpu = port_value, port_step_s, "port", port
        extrap = {"formula": "seconds per solve = median pass wall time x full_rows / sample_rows / processes",
                  "sample_rows": rows_p, "full_rows": full_rows, "processes": n_proc, "interpreter_unavailable": why}
        steps, warmup = args.steps, args.warmup
    else:
        step_s, value = per_step(interp["solve_s_extrapolated"])
        kind = "reference"
        cpu = {"value": value, "unit": unit, "cores": n_proc, "kind": "reference",
               "sample": f"the reference's kbench.runtime forward+backward over its Triton kernels under "
                         f"TRITON_INTERPRET=1 (baseline/_ref), a {interp['sample_rows']}-row family on the "
                         f"config-{args.config} species tree (S={S}), {n_proc} processes at once, {what}"}
        extrap = {"formula": "seconds per solve = median per-process solve time x full_rows / sample_rows / processes",
                  "sample_rows": interp["sample_rows"], "full_rows": full_rows, "processes": n_proc,
                  "sample_solve_s_median": interp["sample_solve_s_median"]}
        steps, warmup = 1, 0
    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "strong" if batched else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator)", "impl": "reference",
        "config": {"workload": f"config{args.config} family, CPU sample", "requested_steps": args.steps,
                   "requested_warmup": args.warmup},
        "extrapolated": extrap,
        "cpu_baseline": cpu,
        "port_secondary": port,
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def per_kernel_arm(args, world, rank):
    """--per-kernel: the reference's glue (``kbench.runtime``) runs one warm-up and one timed pass
    over the reference's own Triton kernels (``baseline/_ref``) and over this project's wrappers
    (a checkout copy whose kernel modules re-export them), each in its own process
    (``baseline/wrapper_bench.py``); one JSON line with both per-wrapper tables."""
    if rank != 0:
        return
    import subprocess
    from baseline import reference
    why = reference.unavailable_reason()
    cfg = 2 if args.config == 3 else args.config  # the micro-bench config of the benchmark text
    if why:
        print(json.dumps({"per_kernel": None, "unavailable": why}), flush=True)
        return
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT / "kernel-bench_b200")
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        roots = {"reference_triton": reference.REF, "ours": reference.checkout_copy(Path(tmp) / "kernel-bench")}
        for name, root in roots.items():
            res = subprocess.run([sys.executable, str(ROOT / "baseline" / "wrapper_bench.py"), "--root", str(root),
                                  "--config", str(cfg)], env=env, capture_output=True, text=True, timeout=1800)
            line = [ln for ln in res.stdout.splitlines() if ln.startswith("WRAPPER_BENCH ")]
            out[name] = json.loads(line[-1].split(" ", 1)[1]) if line else {"error": res.stderr[-2000:]}
    ratio = {}
    ref_w, our_w = out["reference_triton"].get("wrappers", {}), out["ours"].get("wrappers", {})
    for k in ref_w:
        if k in our_w and our_w[k]["ms"] > 0:
            ratio[k] = round(ref_w[k]["ms"] / our_w[k]["ms"], 2)
    print(json.dumps({"per_kernel": True, "config": cfg, "driver": "reference glue (kbench.runtime), one timed pass",
                      "reference_triton": out["reference_triton"], "ours": out["ours"],
                      "speedup_per_wrapper": ratio}), flush=True)


def reference_triton_leg(cap, dev, our_value, steps=2):
    """The unmodified reference's own Triton path (``baseline/_ref``: its stock ``kbench.runtime``
    over its stock kernels) on the same problem and GPU, after this arm's measurements: median
    forward / backward ms of ``steps`` solves after one warm-up solve (which includes Triton's JIT
    compilation), CUDA events.  Not part of ``value``; the ratio is ``speedup``."""
    import torch
    from baseline import parity, reference
    why = reference.unavailable_reason()
    if why:
        return {"unavailable": why}
    t = parity.reference_timing(reference.stock_runtime(), cap, dev, steps)
    torch.cuda.empty_cache()
    return {"solves_per_s": round(t["solves_per_s"], 4), "ms_per_solve": round(t["ms_per_solve"], 1),
            "fwd_ms": round(t["fwd_ms"], 1), "bwd_ms": round(t["bwd_ms"], 1), "steps": steps,
            "first_solve_ms": round(t["first_solve_ms"], 1), "speedup": round(our_value / t["solves_per_s"], 2),
            "what": "reference kbench.runtime.run_forward + run_backward (stock Triton kernels, default options "
                    "of the captured problem), same generated family, same GPU"}


def roofline_from_timers(timers, peak, peak_kind, steps):
    """Dominant level kernel over (static, timer) pairs: algorithmic bytes / device time."""
    from kbench_b200 import engine
    k_ms, k_n, k_bytes = {}, {}, {}
    for static, timer in timers:
        plan = engine.build_plan(static)
        fwd_b, bwd_b = algorithmic_bytes(plan, int(static.state_helpers["S"]))
        for name, (ms, n, per) in timer.totals().items():
            if n == 0:
                continue
            k_ms[name] = k_ms.get(name, 0.0) + ms / steps
            k_n[name] = k_n.get(name, 0) + n / steps
            k_bytes[name] = k_bytes.get(name, 0.0) + kernel_bytes(name, per, fwd_b, bwd_b) / steps
    dominant = max(k_ms, key=k_ms.get)
    achieved = k_bytes[dominant] / (k_ms[dominant] * 1e-3) / 1e9
    return {
        "bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
        "algorithmic_bytes_per_launch": k_bytes[dominant] / k_n[dominant],
        "avg_launch_ms": k_ms[dominant] / k_n[dominant],
        "kernel_ms_per_step": {k: round(v, 3) for k, v in k_ms.items()},
    }


def batch_setup(world, rank, local, n_total, chunk, host_builder=False):
    """This rank's share of the batched workload (config 4): its contiguous block of families, as
    chunks of at most ``chunk`` families -- gene topologies sampled by a spawn pool sized to this
    rank's share of the host's CPUs, the static layouts and the engine's schedules built on the
    device (``host_builder``: the whole generator on the host pool, the schedules on the host)."""
    import torch
    import torch.distributed as dist
    from kbench_b200 import batch, builder

    dev = torch.device("cuda", local if world > 1 else 0)
    f0, f1 = batch.family_block(n_total, world, rank)
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    workers = max(1, len(os.sched_getaffinity(0)) // max(1, local_world))
    t0 = time.perf_counter()
    if host_builder:
        chunks, gen_t = batch.build_chunks(4, f0, f1, chunk, workers=workers), {}
    else:  # gene topologies sampled on the host, layouts built on the device
        chunks, gen_t = builder.generate_chunks(4, f0, f1, chunk, device=dev, workers=workers)
    gen_s = time.perf_counter() - t0
    allreduce = (lambda t: dist.all_reduce(t)) if world > 1 else None
    t0 = time.perf_counter()
    fb = batch.FamilyBatch(chunks, n_total, batch.EngineSolver(dev), allreduce=allreduce)
    load_s = time.perf_counter() - t0
    theta = torch.as_tensor(chunks[0]["inputs"]["theta"]).to(dev)
    cw = torch.as_tensor(chunks[0]["inputs"]["col_weights"]).to(dev)
    S = int(chunks[0]["meta"]["S"])
    info = {"f0": f0, "f1": f1, "rows": fb.rows, "n_chunks": len(chunks), "S": S, "generation_s": round(gen_s, 2),
            "load_s": round(load_s, 2), "layout_builder": "host" if host_builder else "device",
            **{k: round(v, 3) for k, v in gen_t.items()}}
    return dev, fb, theta, cw, info


def batch_timed(fb, theta, cw, dev, world, warmup, steps, *, on_timed_start=None, sampler=None):
    """Device-timed steps of a family batch (barrier + synchronize on both sides; ``on_timed_start``
    runs after the warm-up); returns (ms per step as the max over ranks, launches, clocks, last
    StepResult)."""
    import torch
    import torch.distributed as dist
    from kbench_b200 import _lib

    for _ in range(warmup):
        fb.step(theta, cw)
    torch.cuda.synchronize()
    if on_timed_start is not None:
        on_timed_start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = sum(_lib.LAUNCHES.values())
    if sampler:
        sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        res = fb.step(theta, cw)
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    launches = sum(_lib.LAUNCHES.values()) - launches0
    ms_t = torch.tensor([ev0.elapsed_time(ev1) / steps], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    return float(ms_t.item()), launches, clocks, res


def static_builder_timing(info, n_fam_local, sample=4):
    """The static builder's share of the batched setup: topology sampling (host pool) and the
    device build of this rank's families, against the host generator's layout stage (clade
    amalgamation + wave assembly of :mod:`kbench_b200.gen`) timed on ``sample`` families and
    scaled per family (the families are drawn independently from the same process)."""
    from kbench_b200 import builder
    species, topo = builder.family_topologies(4, n_families=sample)
    t0 = time.perf_counter()
    builder.host_reference(topo, species)
    host_per_family = (time.perf_counter() - t0) / sample
    dev_s = info.get("device_build_s")
    return {"families": n_fam_local, "topology_sampling_s": info.get("sampling_s"),
            "device_layout_s": dev_s, "device_schedule_s": info["load_s"],
            "host_layout_s_per_family": round(host_per_family, 4),
            "host_layout_s_extrapolated": round(host_per_family * n_fam_local, 1),
            "layout_speedup_vs_host": round(host_per_family * n_fam_local / dev_s, 1) if dev_s else None,
            "host_sample": f"{sample} families timed on one host core, scaled per family"}


def config4_strong(args, world, rank, local, warmup=1, steps=3):
    """The batched workload (config 4: ``--families``, default all 1,024, S = 1,023) strong-scaled
    over the N ranks of this run -- each rank owns a contiguous block of families, one all-reduce
    of [loss, 8 x S accumulators] per step -- as a compact object for the headline line (a fixed
    1 warm-up + 3 timed steps, so its cost does not grow with --steps)."""
    import torch
    from kbench_b200 import gen
    n_total = int(args.families or gen.CONFIGS[4].n_families)
    dev, fb, theta, cw, info = batch_setup(world, rank, local, n_total, args.chunk, args.host_builder)
    ms, launches, _, res = batch_timed(fb, theta, cw, dev, world, warmup, steps)
    out = {"workload": f"config4: {n_total} families (S={info['S']}) in contiguous blocks over {world} rank(s), "
                       f"chunks of <= {args.chunk}; one all-reduce of [loss, 8*S accumulators] per step",
           "families": n_total, "families_per_s": round(n_total * 1000.0 / ms, 3), "ms_per_step": round(ms, 3),
           "steps": steps, "warmup": warmup, "scaling": "strong", "rank0_rows": info["rows"],
           "rank0_generation_s": info["generation_s"], "rank0_load_s": info["load_s"],
           "gpu_launches_rank0": int(launches), "loss": float(res.loss)}
    if not args.host_builder and rank == 0:
        out["static_builder"] = static_builder_timing(info, n_fam_local=info["f1"] - info["f0"])
    del fb
    torch.cuda.empty_cache()
    return out


def batch_arm(args, world, rank, local):
    """--config 4: families/s of the batched workload (chunked per GPU, sharded across ranks)."""
    import torch
    import torch.distributed as dist
    from kbench_b200 import engine, gen

    n_total = int(args.families or gen.CONFIGS[4].n_families)
    dev, fb, theta, cw, info = batch_setup(world, rank, local, n_total, args.chunk, args.host_builder)
    f0, f1, rows, n_chunks, S = info["f0"], info["f1"], info["rows"], info["n_chunks"], info["S"]
    gen_s, load_s = info["generation_s"], info["load_s"]
    timers = [(st, engine.LevelTimer()) for st in fb.statics]

    def attach():
        for st, tm in timers:
            st._level_timer = tm

    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    ms_max, launches, clocks, res = batch_timed(fb, theta, cw, dev, world, args.warmup, args.steps,
                                                on_timed_start=attach, sampler=sampler)
    peak, peak_kind = measured_peak()
    roofline = roofline_from_timers(timers, peak, peak_kind, args.steps) if rank == 0 else None
    for st, _ in timers:
        st._level_timer = None

    # end to end: theta / col_weights from pinned host memory, loss + gradients back every step
    n_out = 1 + 3 * S + S
    th_host, cw_host = theta.cpu().pin_memory(), cw.cpu().pin_memory()
    out_host = torch.empty((n_out,), dtype=torch.float64).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        r = fb.step(th_host.to(dev, non_blocking=True), cw_host.to(dev, non_blocking=True))
        out_host.copy_(torch.cat([r.loss.reshape(1), r.grad_theta.reshape(-1).double(),
                                  r.grad_col.reshape(-1).double()]), non_blocking=True)
        torch.cuda.current_stream().synchronize()
        float(out_host[0])
    e1.record()
    torch.cuda.synchronize()
    e_t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e_ms = float(e_t.item())
    if rank == 0:
        line = {
            "metric": "fwd+bwd families/sec (batched config 4: S=1023, ~16k rows per family, shared theta)",
            "value": round(n_total * 1000.0 / ms_max, 3), "unit": "families/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded generator of the benchmark's config text)",
            "config": {
                "workload": f"config4: {n_total} families (S={S}); rank 0 holds families [{f0},{f1}) "
                            f"= {rows} rows in {n_chunks} chunks of <= {args.chunk}",
                "parallelism": f"dp{world} (family blocks), one all-reduce of [loss, 8*S accumulators] per step",
                "l2": "state arrays far larger than L2; no flush needed",
                "generation_s": round(gen_s, 2), "load_s": round(load_s, 2),
                "layout_builder": info["layout_builder"],
            },
            "roofline": roofline, "cpu_baseline": None,
            "e2e": {"value": round(n_total * 1000.0 / e_ms, 3), "unit": "families/s",
                    "h2d_bytes_per_step": int((theta.numel() + cw.numel()) * 4),
                    "d2h_bytes_per_step": int(n_out * 8)},
            "gpu_launches": int(launches), "clocks": clocks,
            "loss": float(res.loss),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def tangent_arm(args, world, rank, local):
    """--config 5: forward + batched forward-mode tangent of the config-3 family (replicas on N>1)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from kbench_b200 import _lib, engine, gen, runtime, tangent

    dev = torch.device("cuda", local if world > 1 else 0)
    cap = gen.generate(5, seed=5000 + rank)
    S, C = int(cap["meta"]["S"]), int(cap["meta"]["C"])
    static = runtime.make_static(cap, dev)
    theta = cap["inputs"]["theta"].to(dev)
    cw = cap["inputs"]["col_weights"].to(dev)
    D = int(args.directions)
    V = torch.from_numpy(np.stack([np.random.Generator(np.random.PCG64(5000 + k)).standard_normal((S, 3))
                                   for k in range(D)]).astype(np.float32)).to(dev)
    plan = engine.build_plan(static)

    def step(th, vv):
        _, saved = runtime.run_forward(static, th, cw)
        return tangent.jvp_batch(static, th, vv, saved)

    for _ in range(args.warmup):
        step(theta, V)
    torch.cuda.synchronize()
    timer = engine.LevelTimer()
    static._level_timer = timer
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = sum(_lib.LAUNCHES.values())
    if sampler:
        sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step(theta, V)
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    launches = sum(_lib.LAUNCHES.values()) - launches0
    totals = timer.totals()
    static._level_timer = None
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # split forward / tangent, and the finite-difference check of two directions
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    _, saved = runtime.run_forward(static, theta, cw)
    ev[1].record()
    roots = tangent.jvp_batch(static, theta, V, saved)
    ev[2].record()
    torch.cuda.synchronize()
    fwd_ms, tan_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    fd_err = []
    eps = 1e-2
    for k in range(2):
        _, sp = runtime.run_forward(static, theta + eps * V[k], cw)
        rp = sp["root_rows"].double()
        del sp
        _, sm_ = runtime.run_forward(static, theta - eps * V[k], cw)
        fd = (rp - sm_["root_rows"].double()) / (2 * eps)
        del sm_
        t = roots[k].double()
        fin = torch.isfinite(fd) & torch.isfinite(t)
        fd_err.append(float((fd[fin] - t[fin]).norm() / fd[fin].norm()))
    del saved, roots

    # end to end: theta and the directions from pinned host memory, root tangents back
    th_host, v_host = theta.cpu().pin_memory(), V.cpu().pin_memory()
    out_host = torch.empty((D, int(static.wave_layout["root_row_ids"].numel()), S), dtype=torch.float32).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for _ in range(args.steps):
        r = step(th_host.to(dev, non_blocking=True), v_host.to(dev, non_blocking=True))
        out_host.copy_(r, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        float(out_host[0, 0, 0])
    x1.record()
    torch.cuda.synchronize()
    x_t = torch.tensor([x0.elapsed_time(x1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(x_t, op=dist.ReduceOp.MAX)
    e_ms = float(x_t.item())
    if rank == 0:
        peak, peak_kind = measured_peak()
        k_ms = {n: v[0] / args.steps for n, v in totals.items() if v[1] > 0}
        tname = "kb_flow_tangent" if "kb_flow_tangent" in k_ms else "kb_level_tangent"
        n_l = totals[tname][1] / args.steps
        # compulsory bytes of the tangent sweep: per direction write dPi, dPibar of every row and
        # read dPi, dPibar of each distinct child once per level; the primal rows once
        kb = sum(4 * S * (D * (2 * (plan.level_ptr[L + 1] - plan.level_ptr[L]) + 2 * plan.children_per_level[L])
                          + 3 * (plan.level_ptr[L + 1] - plan.level_ptr[L]))
                 for L in range(plan.n_levels))
        ach = kb / (k_ms[tname] * 1e-3) / 1e9
        line = {
            "metric": f"fwd + {D}-direction tangent passes/sec (S=4095, C~131k; BASELINE tangent config)",
            "value": round(world * 1000.0 / ms_max, 4), "unit": "passes/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded generator; v ~ N(0,1), seeds 5000+k)",
            "config": {"workload": f"config5: S={S}, C={C} rows, forward + {D} tangent directions "
                                   f"(self_iters = pi_iters = {static.solver_options.pi_iters})",
                       "parallelism": f"replicas x{world}",
                       "l2": "state arrays far larger than L2; no flush needed"},
            "fwd_ms": round(fwd_ms, 3), "tangent_ms": round(tan_ms, 3),
            "fd_check": {"eps": eps, "rel_err": fd_err, "tolerance": 1e-3},
            "roofline": {"bound": "hbm", "kernel": tname, "achieved": round(ach, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(ach / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": None, "algorithmic_bytes_per_launch": kb / n_l,
                         "avg_launch_ms": k_ms[tname] / n_l,
                         "kernel_ms_per_step": {k2: round(v, 3) for k2, v in k_ms.items()}},
            "cpu_baseline": None,
            "e2e": {"value": round(world * 1000.0 / e_ms, 4), "unit": "passes/s",
                    "h2d_bytes_per_step": int((theta.numel() + V.numel()) * 4),
                    "d2h_bytes_per_step": int(out_host.numel() * 4)},
            "gpu_launches": int(launches), "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        reference_arm(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.traffic_case:
        traffic_case(args)
        return
    if args.per_kernel:
        per_kernel_arm(args, world, rank)
        return
    if args.hvp:
        hvp_arm(args, world, rank, local)
        return
    if args.config == 4:
        batch_arm(args, world, rank, local)
        return
    if args.config == 5:
        tangent_arm(args, world, rank, local)
        return
    import torch
    import torch.distributed as dist
    from kbench_b200 import _lib, engine, gen, runtime

    dev = torch.device("cuda", local if world > 1 else 0)
    seed = 1000 * args.config + rank
    cap = gen.generate(args.config, seed=seed)
    S = int(cap["meta"]["S"])
    C = int(cap["meta"]["C"])
    static = runtime.make_static(cap, dev)
    static._deterministic_backward = not args.atomic_backward
    theta = cap["inputs"]["theta"].to(dev)
    cw = cap["inputs"]["col_weights"].to(dev)
    plan = engine.build_plan(static)
    fwd_b, bwd_b = algorithmic_bytes(plan, S)
    n_grad = 1 + 3 * S + S

    def allreduce(loss, gt, gc):
        if world > 1:
            packed = torch.cat([loss.reshape(1).float(), gt.reshape(-1).float(), gc.reshape(-1).float()])
            dist.all_reduce(packed)
            return packed
        return None

    def step(th, c, check=True):
        # the solve's one host synchronisation (the dataflow error check) at the end of the
        # backward, or -- check=False, in the device-timed loop -- once after the loop
        loss, saved = runtime.run_forward(static, th, c, check_errors=False)
        gt, gc = runtime.run_backward(static, th, c, saved, check_errors=check)
        allreduce(loss, gt, gc)
        return loss, gt, gc

    for _ in range(args.warmup):
        step(theta, cw)
    torch.cuda.synchronize()

    # ---- device-timed region (inputs resident; state arrays far larger than L2) ----
    timer = engine.LevelTimer()
    static._level_timer = timer
    sampler = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = sum(_lib.LAUNCHES.values())
    if sampler:
        sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        step(theta, cw, check=False)
    t_end.record()
    torch.cuda.synchronize()
    runtime.check_errors(static)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    launches = sum(_lib.LAUNCHES.values()) - launches0
    ms = t_start.elapsed_time(t_end) / args.steps
    totals = timer.totals()
    static._level_timer = None
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # ---- split forward / backward time (one extra untimed-for-value pass) ----
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    loss, saved = runtime.run_forward(static, theta, cw)
    ev[1].record()
    runtime.run_backward(static, theta, cw, saved)
    ev[2].record()
    torch.cuda.synchronize()
    fwd_ms, bwd_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])

    # ---- end-to-end through the public API with host buffers ----
    del loss, saved  # the split pass's saved state: e2e steps reuse the same cached blocks
    th_host = theta.detach().cpu().pin_memory()
    cw_host = cw.detach().cpu().pin_memory()
    out_host = torch.empty((n_grad,), dtype=torch.float32).pin_memory()

    def e2e_step():
        th_d = th_host.to(dev, non_blocking=True)
        cw_d = cw_host.to(dev, non_blocking=True)
        loss, gt, gc = step(th_d, cw_d)
        res = torch.cat([loss.reshape(1).float(), gt.reshape(-1).float(), gc.reshape(-1).float()])
        out_host.copy_(res, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return float(out_host[0])

    e2e_step()  # untimed: first use of the pinned buffers on this path
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        e2e_step()
    e_end.record()
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_end) / args.steps
    e_t = torch.tensor([e_ms], device=dev)
    if world > 1:
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e_ms = float(e_t.item())

    # ---- the batched workload (config 4), strong-scaled over the same ranks ----
    config4 = None
    if not args.no_config4:
        torch.cuda.empty_cache()
        config4 = config4_strong(args, world, rank, local)

    if rank == 0:
        peak, peak_kind = measured_peak()
        k_tot = {name: v[0] / args.steps for name, v in totals.items()}
        dominant = max(k_tot, key=k_tot.get)
        per = totals[dominant][2]
        alg_bytes = kernel_bytes(dominant, per, fwd_b, bwd_b) / args.steps
        k_ms = k_tot[dominant]
        achieved = alg_bytes / (k_ms * 1e-3) / 1e9
        n_launch = totals[dominant][1] / args.steps
        roofline = {
            "bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1), "peak": peak,
            "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
            "traffic": None,
            "algorithmic_bytes_per_launch": alg_bytes / n_launch,
            "avg_launch_ms": k_ms / n_launch,
            "kernel_ms_per_step": {k: round(v, 3) for k, v in k_tot.items() if v > 0},
        }
        # per dataflow kernel: HBM fraction of the algorithmic bytes and, where captured for this
        # build, DRAM traffic and the issue-slot bound (warp instructions at the sampled clock)
        smx = (clocks or {}).get("sm_mhz") or 1965.0
        per_kernel = {}
        for name, kms in k_tot.items():
            if kms <= 0 or not name.startswith("kb_flow_"):
                continue
            kb = sum((fwd_b if "forward" in name else bwd_b).values())
            entry = {"ms": round(kms, 3), "hbm_gbs": round(kb / (kms * 1e-3) / 1e9, 1),
                     "hbm_frac": round(kb / (kms * 1e-3) / 1e9 / peak, 4), "algorithmic_bytes": kb}
            cnt = launch_counters(name, C, S, None if name != "kb_flow_backward" else
                                  ("deterministic" if getattr(static, "_edge_scratch", None) is not None
                                   else "atomic"))
            if cnt is not None:
                entry["dram_bytes"] = cnt["dram_read"] + cnt["dram_write"]
                entry["dram_over_algorithmic"] = round(entry["dram_bytes"] / kb, 3)
                if cnt.get("warp_inst"):
                    entry["issue"] = issue_roofline(cnt["warp_inst"], kms, smx)
            per_kernel[name] = entry
        roofline["per_kernel"] = per_kernel
        dom = per_kernel.get(dominant, {})
        if "dram_bytes" in dom:
            roofline["traffic"] = dom["dram_bytes"]
            roofline["traffic_note"] = ("dram__bytes_read.sum + dram__bytes_write.sum of one full-size launch on "
                                        "this family (single-pass ncu capture of bench.py --traffic-case config3)")
        if "issue" in dom:
            roofline["issue_bound"] = dom["issue"]
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            sps, dt, rows = run_cpu_oracle_sample(C, seed=3000)
            cpu = {"value": sps, "unit": "solves/s", "cores": 1, "kind": "port",
                   "sample": f"numpy oracle fwd+bwd of a {rows}-row family on the config-3 species tree "
                             f"(S={S}), {dt:.1f} s, extrapolated per row to C={C}"}
        value = world * 1000.0 / ms_max
        ref_triton = None
        if world == 1 and not args.no_reference_triton:
            ref_triton = reference_triton_leg(cap, dev, value)
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "solves/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded generator of the benchmark's config text)",
            "config": {
                "workload": f"config{args.config}: S={S}, C={C} rows, {plan.n_splits} splits, "
                            f"{len(static.wave_layout['wave_metas'])} size-waves -> {plan.n_levels} dependency "
                            f"levels, pi_iters={static.solver_options.pi_iters}, "
                            f"neumann_terms={static.solver_options.neumann_terms}; one family per GPU, "
                            "gradients all-reduced",
                "parallelism": f"dp{world} (families)",
                "l2": "state arrays (C*S*4 bytes each) far larger than L2; no flush needed",
                "backward": ("deterministic (edge rows)" if getattr(static, "_edge_scratch", None) is not None
                             else "atomic child adds"),
            },
            "ms_per_solve": round(ms_max, 3), "fwd_ms": round(fwd_ms, 3), "bwd_ms": round(bwd_ms, 3),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "reference_triton": ref_triton,
            "config4": config4,
            "e2e": {"value": round(world * 1000.0 / e_ms, 4), "unit": "solves/s",
                    "h2d_bytes_per_step": int(theta.numel() * 4 + cw.numel() * 4),
                    "d2h_bytes_per_step": int(n_grad * 4)},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
