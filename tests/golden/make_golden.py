"""Generate the golden fixtures that pin the CPU oracle to the reference itself.

Runs ONLY in a container that has the reference project checked out (pass its root with
``--reference``); the outputs are small ``.npz`` files committed beside this script, so nothing at
test time needs the reference.

What it does, per case:
  1. builds a problem with ``kbench_b200.gen`` (seeded, config-1 sized or smaller);
  2. imports the reference's ``kbench`` package with its *pristine* kernels
     (``experiments/pristine_kernels/*`` -- the kernels the reference uses to produce its own
     goldens, ``capture/capture.py:1-19``) swapped in for ``kbench.core.kernels.*``, and runs
     them on the CPU under ``TRITON_INTERPRET=1``.  Two CUDA-only guards of the pristine backward
     (``wave_backward.py:166-201`` ``active_mask_from_rhs_absmax_fused`` and ``:1001-1002``
     ``_wave_backward_uniform_2d``) are relaxed in memory (the source files are not modified and
     not copied);
  3. runs the reference's unchanged ``kbench.runtime.run_forward`` and ``run_backward`` (the
     backward fed the forward's own intermediates, as ``bench/backward.py`` does);
  4. saves the static layout, the inputs and every checked output.

Usage:  python tests/golden/make_golden.py --reference <path-to-reference-checkout>
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "kernel-bench_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from kbench_b200 import gen  # noqa: E402
from kbench_b200.problem_io import flatten_case  # noqa: E402


def _load_module(name: str, path: Path, patches=()):
    src = path.read_text()
    for old, new in patches:
        if old not in src:
            raise RuntimeError(f"patch anchor not found in {path}: {old!r}")
        src = src.replace(old, new)
    mod = types.ModuleType(name)
    mod.__file__ = str(path)
    sys.modules[name] = mod
    exec(compile(src, str(path), "exec"), mod.__dict__)
    return mod


def install_pristine(ref: Path):
    sys.path.insert(0, str(ref))
    import kbench.core.kernels  # noqa: F401  (package object)
    pk = ref / "experiments" / "pristine_kernels"
    _load_module("kbench.core.kernels._dts_layout_contract", pk / "_dts_layout_contract.py")
    _load_module("kbench.core.kernels.dts_fused", pk / "dts_fused.py")
    _load_module("kbench.core.kernels.e_step", pk / "e_step.py")
    _load_module("kbench.core.kernels.wave_step", pk / "wave_step.py")
    _load_module(
        "kbench.core.kernels.wave_backward", pk / "wave_backward.py",
        patches=[
            ('if rhs.device.type != "cuda":', "if False:"),
            ('if Pi_star.device.type != "cuda":', "if False:"),
        ],
    )
    from kbench import runtime
    return runtime


CASES = {
    # name: (config or ProblemConfig, seed, solver option overrides)
    "small_s1000": (1, 1000, {}),
    "small_s1001_defaults": (1, 1001, {"pi_iters": 6, "neumann_terms": 3}),
    "tiny_s7": (gen.ProblemConfig("tiny", 4, 6, 3, 4, 12), 7, {}),
    "twofam_s31": (gen.ProblemConfig("twofam", 16, 20, 4, 10, 60, n_families=2), 31,
                   {"pi_iters": 4, "neumann_terms": 5}),
}


def run_case(runtime, name, cfg, seed, overrides):
    cap = gen.generate(cfg, seed=seed, solver_options=overrides)
    static = runtime.make_static(cap, "cpu")
    theta = cap["inputs"]["theta"]
    cw = cap["inputs"]["col_weights"]
    t0 = time.time()
    loss, saved = runtime.run_forward(static, theta, cw)
    t1 = time.time()
    g_theta, g_col = runtime.run_backward(static, theta, cw, saved)
    t2 = time.time()
    out = {
        "loss": np.asarray(float(loss), dtype=np.float32),
        "grad_theta": g_theta.detach().numpy(),
        "grad_col": g_col.detach().numpy(),
    }
    for k, v in saved.items():
        out[k] = v.detach().numpy()
    arrays = flatten_case(cap, out)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"[{name}] S={cap['meta']['S']} C={cap['meta']['C']} waves={cap['meta']['n_waves']} "
          f"loss={float(loss):.6f} fwd {t1 - t0:.1f}s bwd {t2 - t1:.1f}s")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--cases", default=",".join(CASES))
    args = ap.parse_args()
    torch.set_num_threads(1)
    runtime = install_pristine(args.reference.resolve())
    for name in args.cases.split(","):
        cfg, seed, ov = CASES[name]
        run_case(runtime, name, cfg, seed, ov)


if __name__ == "__main__":
    main()
