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

Tangent fixtures (``--tangent``): for each forward fixture already in this folder, the
reference's forward-mode tangent ``newton/forward_tangent.py`` ``jvp_root_scores`` (its own
``kbench/core/kernels/{e_step_tangent,dts_tangent,wave_tangent}.py`` kernels, fused fixed-count
self-loop with ``self_iters = pi_iters``), evaluated at the fixture's saved forward intermediates
along two seeded directions ``v ~ N(0,1)`` of theta's shape (seed 5000 + k); saved as
``tangent/<case>.npz``.

HVP fixtures (``--hvp``): for each forward fixture, the reference's analytic exact-Hessian HVP
``newton/hvp_exact.py`` ``make_exact_hvp`` (its own ``kbench/core/kernels/{wave_so,dts_so,
e_step_so}.py`` second-order kernels over the pristine first-order ones) at the fixture's saved
forward intermediates along the same two seeded directions, with the driver's debug tangents
(``d_g*`` accumulators, the E-side rhs ``dq_E`` and solve ``dwE``); saved as ``hvp/<case>.npz``.

Usage:  python tests/golden/make_golden.py --reference <path-to-reference-checkout> [--tangent | --hvp]
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
    # S = 79: a padded width (96) that is not a multiple of 128 columns
    "odd_s79": (gen.ProblemConfig("odd79", 40, 16, 3, 8, 0), 79, {}),
    # non-uniform column weights (col_weights ~ N(0,1), seed 77): the weighted column path
    "weighted_s31": (gen.ProblemConfig("weighted", 16, 20, 4, 10, 0), 3131, {"_col_weights_seed": 77}),
    # the other adjoint options: no activity pruning, and a Pibar-side activity threshold
    "options_s63": (1, 6363, {"use_adjoint_pruning": False, "pibar_side_threshold": 1e-3}),
    # the GMRES self-loop solver (neumann_terms = Arnoldi steps per wave)
    "gmres_s64": (1, 6464, {"self_loop_solver": "gmres", "neumann_terms": 8}),
    # the backward's convergence diagnostics (collect_backward_relres: per family the largest
    # |last Neumann term| / |v| and |v|), on a two-family problem
    "relres_s32": (gen.ProblemConfig("relres", 16, 20, 4, 10, 60, n_families=2), 3232,
                   {"pi_iters": 6, "neumann_terms": 4, "_collect_relres": True}),
    # rates off the benchmark distribution (theta columns shifted by (dup, loss, transfer) log2-odds):
    # rows whose values span more than 100 binades (the forward kernels' per-row log-space
    # recomputation), with every linear constant still >= 2^-26
    "rowfallback_s63": (gen.ProblemConfig("y", 32, 48, 8, 80, 300), 11, {"_theta_shift": (0.0, 5.0, -10.0)}),
    # transfer 2^-30 below the benchmark's: constants below 2^-26, every row in log space
    "forcelog_s31": (gen.ProblemConfig("x", 16, 24, 4, 20, 60), 11,
                     {"pi_iters": 6, "neumann_terms": 4, "_theta_shift": (0.0, 0.0, -30.0)}),
}


def run_case(runtime, name, cfg, seed, overrides):
    overrides = dict(overrides)
    cw_seed = overrides.pop("_col_weights_seed", None)
    collect_relres = overrides.pop("_collect_relres", False)
    theta_shift = overrides.pop("_theta_shift", None)
    cap = gen.generate(cfg, seed=seed, solver_options=overrides)
    if theta_shift is not None:
        cap["inputs"]["theta"] = cap["inputs"]["theta"] + torch.tensor(theta_shift, dtype=torch.float32)
    if cw_seed is not None:
        S = int(cap["meta"]["S"])
        w = np.random.Generator(np.random.PCG64(cw_seed)).standard_normal(S).astype(np.float32)
        cap["inputs"]["col_weights"] = torch.from_numpy(w)
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
    if collect_relres:
        relres, vk_mag = backward_relres(static, theta, cw, saved)
        out["relres"] = relres.detach().numpy()
        out["vk_mag"] = vk_mag.detach().numpy()
    arrays = flatten_case(cap, out)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"[{name}] S={cap['meta']['S']} C={cap['meta']['C']} waves={cap['meta']['n_waves']} "
          f"loss={float(loss):.6f} fwd {t1 - t0:.1f}s bwd {t2 - t1:.1f}s")


def backward_relres(static, theta, cw, saved):
    """The reference glue's backward with ``collect_backward_relres=True`` (same arguments as
    ``kbench/runtime.py:77-115`` passes): per family (relres, vk_mag)."""
    from kbench.api._implicit_grad import implicit_grad_loglik_vjp_wave
    from kbench.core.inference.solver import col_weights_are_uniform
    so = static.solver_options
    return implicit_grad_loglik_vjp_wave(
        static.wave_layout, static.state_helpers, Pi_star_wave=saved["pi_wave"],
        Pibar_star_wave=saved["pibar_wave"], E_star=saved["E"], Ebar=saved["Ebar"], E_s1=saved["E_s1"],
        E_s2=saved["E_s2"], log_pS=saved["log_pS"], log_pD=saved["log_pD"], log_pL=saved["log_pL"],
        max_coupling_mat=saved["max_coupling"], col_log_probs=saved["col_log_probs"],
        use_col_weights=not col_weights_are_uniform(cw), theta=theta, col_weights=cw,
        item_idx=static.rate_item_idx, uniform_pibar_row_max=saved["pibar_row_max"], statewise=static.statewise,
        itemwise=static.itemwise, neumann_terms=so.neumann_terms, self_loop_solver=so.self_loop_solver,
        bicgstab_max_iter=so.bicgstab_max_iter, bicgstab_tol=so.bicgstab_tol,
        bicgstab_breakdown_tol=so.bicgstab_breakdown_tol, adjoint_pruning_threshold=so.adjoint_pruning_threshold,
        use_adjoint_pruning=so.use_adjoint_pruning, pibar_side_threshold=so.pibar_side_threshold,
        collect_backward_relres=True)


TANGENT_DIRECTIONS = 2


def tangent_direction(S: int, k: int) -> np.ndarray:
    """Seeded tangent direction ``v ~ N(0,1)`` of theta's shape [S,3] (seed 5000 + k)."""
    rng = np.random.Generator(np.random.PCG64(5000 + k))
    return rng.standard_normal((S, 3)).astype(np.float32)


def run_tangent_case(runtime, name):
    from kbench_b200.problem_io import unflatten_case
    from newton.forward_tangent import jvp_root_scores
    cap, out = unflatten_case(np.load(HERE / f"{name}.npz"))
    cap = gen.to_torch(cap)
    static = runtime.make_static(cap, "cpu")
    theta = cap["inputs"]["theta"]
    S = int(theta.shape[0])
    sv = {k: torch.from_numpy(np.asarray(v)) for k, v in out.items() if k not in ("loss", "grad_theta", "grad_col")}
    iters = int(cap["meta"]["solver_options"]["pi_iters"])
    arrays = {}
    t0 = time.time()
    for k in range(TANGENT_DIRECTIONS):
        v = torch.from_numpy(tangent_direction(S, k))
        roots, full = jvp_root_scores(static, theta, v, sv, self_iters=iters, return_full=True)
        arrays[f"v{k}"] = v.numpy()
        arrays[f"roots{k}"] = roots.numpy()
        arrays[f"dPi{k}"] = full["dPi"].numpy()
        arrays[f"dPibar{k}"] = full["dPibar"].numpy()
        for key in ("dE", "dE_s1", "dE_s2", "dEbar", "dlog_pS", "dlog_pD", "dlog_pL", "dmax_coupling"):
            arrays[f"{key}{k}"] = full[key].reshape(-1).numpy()
    (HERE / "tangent").mkdir(exist_ok=True)
    np.savez_compressed(HERE / "tangent" / f"{name}.npz", self_iters=np.asarray(iters), **arrays)
    print(f"[tangent {name}] S={S} directions={TANGENT_DIRECTIONS} {time.time() - t0:.1f}s")


HVP_DIRECTIONS = 2
HVP_DEBUG_KEYS = ("d_gE", "d_gpD", "d_gpS", "d_gmc", "d_gEbar", "d_gEs1", "d_gEs2", "dq_E", "dwE")


def run_hvp_case(runtime, name):
    """The reference's analytic exact-Hessian HVP (``newton/hvp_exact.py`` ``make_exact_hvp``:
    point cache from the production backward, tangent forward with ``self_iters = pi_iters``,
    tangent-adjoint sweep with ``wave_so`` / ``dts_so`` / ``e_step_so``, smooth parameter head),
    at the fixture's saved forward intermediates, along the tangent fixtures' directions."""
    from kbench_b200.problem_io import unflatten_case
    from newton.hvp_exact import make_exact_hvp
    cap, out = unflatten_case(np.load(HERE / f"{name}.npz"))
    cap = gen.to_torch(cap)
    static = runtime.make_static(cap, "cpu")
    theta = cap["inputs"]["theta"]
    cw = cap["inputs"]["col_weights"]
    S = int(theta.shape[0])
    sv = {k: torch.from_numpy(np.asarray(v)) for k, v in out.items() if k not in ("loss", "grad_theta", "grad_col")}
    arrays = {}
    t0 = time.time()
    dbg: dict = {}
    hvp = make_exact_hvp(static, theta, cw, sv, debug_out=dbg)
    for k in range(HVP_DIRECTIONS):
        u = torch.from_numpy(tangent_direction(S, k)).reshape(-1)
        dbg.clear()
        hu = hvp(u)
        arrays[f"u{k}"] = u.numpy()
        arrays[f"hu{k}"] = hu.detach().numpy()
        for key in HVP_DEBUG_KEYS:
            arrays[f"{key}{k}"] = dbg[key].reshape(-1).numpy()
    (HERE / "hvp").mkdir(exist_ok=True)
    np.savez_compressed(HERE / "hvp" / f"{name}.npz", **arrays)
    print(f"[hvp {name}] S={S} directions={HVP_DIRECTIONS} {time.time() - t0:.1f}s")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--cases", default=",".join(CASES))
    ap.add_argument("--tangent", action="store_true", help="tangent fixtures from the forward fixtures")
    ap.add_argument("--hvp", action="store_true", help="exact-Hessian HVP fixtures from the forward fixtures")
    args = ap.parse_args()
    torch.set_num_threads(1)
    runtime = install_pristine(args.reference.resolve())
    for name in args.cases.split(","):
        if args.hvp:
            run_hvp_case(runtime, name)
        elif args.tangent:
            run_tangent_case(runtime, name)
        else:
            cfg, seed, ov = CASES[name]
            run_case(runtime, name, cfg, seed, ov)


if __name__ == "__main__":
    main()
