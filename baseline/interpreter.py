"""The reference's own implementation on the host CPU (BASELINE B3): its stock ``kbench.runtime``
over its stock Triton kernels (``baseline/_ref``), run by Triton's interpreter
(``TRITON_INTERPRET=1``) on CPU tensors.

Two CUDA-only guards of the reference's backward (``kbench/core/kernels/wave_backward.py``:
``active_mask_from_rhs_absmax_fused`` and ``_wave_backward_uniform_2d`` raise unless their inputs
are on a CUDA device) are relaxed in memory when the module is loaded; the source files are
neither modified nor copied.  Everything else is the installed reference, unchanged.

Each solve runs in its own ``spawn`` process (the interpreter executes one program at a time, so a
process is one core); ``parallel`` starts ``n`` of them together and returns each one's wall time.

    python baseline/interpreter.py --config 1            # one full config-1 solve
    python baseline/interpreter.py --sample-genes 8 -n 16
"""

from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import sys
import time
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
GUARDS = [('if rhs.device.type != "cuda":', "if False:"), ('if Pi_star.device.type != "cuda":', "if False:")]


def unavailable_reason() -> str | None:
    """Why the reference cannot run under the interpreter here (None when it can; no GPU needed)."""
    from baseline import reference
    if not reference.available():
        return "reference not installed in baseline/_ref (python baseline/reference.py --install <checkout>)"
    try:
        import triton  # noqa: F401
    except Exception as exc:  # noqa: BLE001
        return f"triton not importable: {exc}"
    return None


def _load_patched(name: str, path: Path):
    src = path.read_text()
    for old, new in GUARDS:
        if old not in src:
            raise RuntimeError(f"guard not found in {path}: {old!r}")
        src = src.replace(old, new)
    mod = types.ModuleType(name)
    mod.__file__ = str(path)
    sys.modules[name] = mod
    exec(compile(src, str(path), "exec"), mod.__dict__)
    return mod


def _problem(spec):
    from kbench_b200 import gen
    kind, value, seed = spec
    if kind == "config":
        return gen.generate(int(value), seed=seed)
    if kind == "tiny":  # 4 species leaves, 6 genes: a seconds-long check of the path
        return gen.generate(gen.ProblemConfig("tiny", 4, 6, 3, 4, 12), seed=seed)
    # a small family on the config-3 species tree: the headline's per-row work, fewer rows
    cfg = gen.ProblemConfig("interp_sample", gen.CONFIGS[3].n_species, int(value), 2, max(8, int(value) // 3), 0,
                            solver_options=dict(gen.CONFIGS[3].solver_options))
    return gen.generate(cfg, seed=seed)


def solve_once(spec) -> dict:
    """One forward + backward of the reference under the interpreter (call in a fresh process)."""
    os.environ["TRITON_INTERPRET"] = "1"
    from baseline import reference
    sys.path.insert(0, str(reference.REF))
    sys.path.insert(1, str(ROOT / "kernel-bench_b200"))
    import torch
    import kbench.core.kernels  # noqa: F401  (the package object the patched module joins)
    _load_patched("kbench.core.kernels.wave_backward", reference.REF / "kbench" / "core" / "kernels" / "wave_backward.py")
    from kbench import runtime
    cap = _problem(spec)
    st = runtime.make_static(cap, torch.device("cpu"))
    theta, cw = cap["inputs"]["theta"], cap["inputs"]["col_weights"]
    t0 = time.perf_counter()
    loss, saved = runtime.run_forward(st, theta, cw)
    t1 = time.perf_counter()
    runtime.run_backward(st, theta, cw, saved)
    t2 = time.perf_counter()
    return {"rows": int(cap["meta"]["C"]), "S": int(cap["meta"]["S"]), "loss": float(loss), "fwd_s": t1 - t0,
            "bwd_s": t2 - t1, "solve_s": t2 - t0}


def parallel(spec, n: int) -> list[dict]:
    """``n`` solves of ``spec`` in ``n`` spawn processes started together."""
    with mp.get_context("spawn").Pool(n) as pool:
        return pool.map(solve_once, [spec] * n, chunksize=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=None)
    ap.add_argument("--sample-genes", type=int, default=8)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("-n", type=int, default=1, help="processes started together")
    a = ap.parse_args()
    spec = ("config", a.config, 1000 * a.config if a.seed is None else a.seed) if a.config else \
        ("sample", a.sample_genes, 3000 if a.seed is None else a.seed)
    res = parallel(spec, a.n)
    print(json.dumps({"spec": spec, "cores": len(os.sched_getaffinity(0)), "processes": a.n, "runs": res}), flush=True)


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    main()
