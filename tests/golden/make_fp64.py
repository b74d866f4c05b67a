"""Generate fp64 evaluations of the benchmark problems (configs 2 and 3) -- the yardstick for the
parity tests that compare the reference's Triton path and this project's kernels at full size.

At full size the reference's fp32 implementation and ours differ by rounding (atomic add order,
fp32 running sums of the gradient columns), and the implicit gradients amplify rounding of the
forward state.  Neither fp32 result is "the" answer, so both are measured against the same
algorithm evaluated in float64: the numpy oracle (``oracle/kb_oracle.py``, which restates the
reference's pristine kernels and glue call by call) loaded at float64 precision
(``kb_oracle.at_precision``), run on the very problem the GPU tests and ``bench.py`` generate
(``gen.generate(config, seed=1000*config)``, seeded, deterministic).

Saved per config in ``fp64/config<N>.npz`` (a few MB): the loss, the E-step vectors, every row's
``pibar_row_max``, the root rows, a seeded sample of Pi / Pibar rows, ``grad_theta`` and
``grad_col``, and the problem's size counters (checked on load so a generator change cannot
silently pair the fixture with another problem).  Runs on the CPU in this container; config 2
takes half a minute, config 3 about an hour and ~30 GB of host memory.

Usage:  python tests/golden/make_fp64.py --config 2 [--config 3]
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
for _p in (REPO, REPO / "kernel-bench_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

from kbench_b200 import gen  # noqa: E402
from oracle import kb_oracle  # noqa: E402

SAMPLE_ROWS = 64


def sample_rows(C: int, roots, seed: int) -> np.ndarray:
    """Seeded sample of row ids (the roots included), sorted."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ids = rng.choice(C, size=min(C, SAMPLE_ROWS), replace=False)
    return np.unique(np.concatenate([ids, np.asarray(roots, dtype=np.int64)])).astype(np.int64)


def problem_counters(cap: dict) -> dict:
    m = cap["meta"]
    wl = cap["static"]["wave_layout"]
    n_splits = sum(int(np.asarray(w["sl"]).shape[0]) for w in wl["wave_metas"] if "sl" in w)
    return {"S": int(m["S"]), "C": int(m["C"]), "n_splits": n_splits, "n_waves": len(wl["wave_metas"])}


def run(config: int) -> None:
    seed = 1000 * config
    t0 = time.time()
    cap = gen.generate(config, seed=seed, as_torch=False)
    cnt = problem_counters(cap)
    print(f"[config {config}] generated S={cnt['S']} C={cnt['C']} splits={cnt['n_splits']} "
          f"({time.time() - t0:.1f}s)", flush=True)
    o64 = kb_oracle.at_precision(np.float64)
    st = dict(cap["static"])
    st["solver_options"] = cap["meta"]["solver_options"]
    theta = cap["inputs"]["theta"].astype(np.float64)
    cw = cap["inputs"]["col_weights"].astype(np.float64)
    t1 = time.time()
    loss, saved = o64.forward(st, theta, cw)
    t2 = time.time()
    print(f"[config {config}] fp64 forward {t2 - t1:.0f}s loss={loss:.10f}", flush=True)
    g_theta, g_col = o64.backward(st, theta, cw, saved, acc_dtype=np.float64)
    t3 = time.time()
    print(f"[config {config}] fp64 backward {t3 - t2:.0f}s", flush=True)
    roots = np.asarray(cap["static"]["wave_layout"]["root_row_ids"], dtype=np.int64)
    rows = sample_rows(cnt["C"], roots, seed + 11)
    out = {
        "seed": np.asarray(seed), **{k: np.asarray(v) for k, v in cnt.items()},
        "loss": np.asarray(loss, dtype=np.float64),
        "E": saved["E"], "E_s1": saved["E_s1"], "E_s2": saved["E_s2"], "Ebar": saved["Ebar"],
        "pibar_row_max": saved["pibar_row_max"], "root_rows": saved["root_rows"],
        "sample_rows": rows, "pi_rows": saved["pi_wave"][rows], "pibar_rows": saved["pibar_wave"][rows],
        "grad_theta": np.asarray(g_theta, dtype=np.float64), "grad_col": np.asarray(g_col, dtype=np.float64),
        "e_iters": np.asarray(saved["e_iters"]),
    }
    (HERE / "fp64").mkdir(exist_ok=True)
    np.savez_compressed(HERE / "fp64" / f"config{config}.npz", **out)
    print(f"[config {config}] saved fp64/config{config}.npz ({time.time() - t0:.0f}s total)", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, action="append", required=True)
    for c in ap.parse_args().config:
        run(c)


if __name__ == "__main__":
    main()
