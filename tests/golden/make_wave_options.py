"""Goldens for the two remaining options of ``wave_backward_uniform_fused``: a warm-started
fixed-point solve (``initial_v``) and gradient accumulation into caller targets
(``self_loop_grad_targets``), produced by the reference's own pristine kernels.

Runs ONLY in a container with the reference checkout (``--reference``).  It swaps the reference's
pristine kernels in for ``kbench.core.kernels.*`` and runs them on the CPU under
``TRITON_INTERPRET=1``, exactly as ``make_golden.py`` does; runs the reference's unchanged glue
(``kbench.runtime.run_forward / run_backward``) on a generated problem while recording every
``wave_backward_uniform_fused`` call the glue makes (its arguments, cloned before the call); takes
the recorded call with the most rows; deactivates a seeded third of its rows (so inactive rows are
exercised); and calls the pristine wrapper again on fresh copies of those arguments with the
options of each case below.  The arguments (once) and every case's options and outputs go to
``wave_options_s64.pt``, a plain dict of CPU tensors and numbers.

Reference semantics recorded here (``kbench/core/kernels/wave_backward.py``):
  * ``initial_v`` (Neumann only, :1493-1534): ``v = initial_v``, then ``neumann_terms`` fixed-point
    updates ``v <- rhs + J_self^T v`` on active rows; inactive rows keep ``initial_v``; no last
    increment (:1596-1600).
  * ``self_loop_grad_targets`` = (grad_log_pD, grad_log_pS, grad_E, grad_Ebar, grad_E_s1,
    grad_E_s2, grad_mt, param_grad_vector) (:1615-1640, the ACCUM_GRADS branch of the parameter
    store, :1213-1262): the column sums over active rows of the buckets are ADDED into the targets
    -- pD += aw0, pS += aw345 (per column, or one scalar sum when param_grad_vector is false),
    E += aw0 + aw2, Ebar += aw1, E_s1 += aw4, E_s2 += aw3, mt += aw2 -- and the six bucket
    outputs are None.

Usage:  python tests/golden/make_wave_options.py --reference <path-to-reference-checkout>
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import make_golden  # noqa: E402  (sets up the package path; install_pristine)
from kbench_b200 import gen  # noqa: E402

OUT = HERE / "wave_options_s64.pt"
CFG = gen.ProblemConfig("waveopts", 16, 24, 4, 12, 60)
SEED = 6464
SOLVER = {"pi_iters": 6, "neumann_terms": 5}
TARGET_NAMES = ("grad_log_pD", "grad_log_pS", "grad_E", "grad_Ebar", "grad_E_s1", "grad_E_s2", "grad_mt")


def _clone(o):
    if torch.is_tensor(o):
        return o.detach().clone()
    if isinstance(o, dict):
        return {k: _clone(v) for k, v in o.items()}
    if isinstance(o, (list, tuple)):
        return type(o)(_clone(v) for v in o)
    return o


def _targets(rng, S, vector):
    n = S if vector else 1
    vals = [torch.from_numpy(rng.standard_normal(n if i < 2 else S).astype(np.float32)) for i in range(7)]
    return vals, bool(vector)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    runtime = make_golden.install_pristine(args.reference.resolve())
    import kbench.api._implicit_grad as ig
    pristine = ig.wave_backward_uniform_fused
    calls = []

    def record(*a, **kw):
        calls.append(_clone((a, kw)))
        return pristine(*a, **kw)

    ig.wave_backward_uniform_fused = record
    cap = gen.generate(CFG, seed=SEED, solver_options=SOLVER)
    static = runtime.make_static(cap, "cpu")
    theta, cw = cap["inputs"]["theta"], cap["inputs"]["col_weights"]
    _, saved = runtime.run_forward(static, theta, cw)
    runtime.run_backward(static, theta, cw, saved)
    ig.wave_backward_uniform_fused = pristine

    a0, kw0 = max(calls, key=lambda c: int(c[0][3]))  # positional W
    W, S = int(a0[3]), int(a0[4])
    rng = np.random.Generator(np.random.PCG64(SEED))
    mask = kw0.get("active_mask")
    mask = torch.ones(W, dtype=torch.bool) if mask is None else mask.clone().reshape(W).bool()
    mask &= torch.from_numpy(rng.random(W) >= 1.0 / 3.0)
    kw0 = dict(kw0)
    kw0["active_mask"] = mask
    rhs = a0[6]
    init_v = torch.from_numpy(rng.standard_normal((W, S)).astype(np.float32)) * rhs.abs().max()

    cases = {
        "initial_v": {"initial_v": init_v, "return_last_increment": True},
        "initial_v_zero_terms": {"initial_v": init_v, "neumann_terms": 0},
        "targets_vector": {"self_loop_grad_targets": _targets(rng, S, True), "return_last_increment": True},
        "targets_scalar": {"self_loop_grad_targets": _targets(rng, S, False)},
        "initial_v_targets": {"initial_v": init_v, "self_loop_grad_targets": _targets(rng, S, True)},
    }
    out = {"args": a0, "kwargs": kw0, "W": W, "S": S, "cases": {}}
    for name, extra in cases.items():
        a, kw = _clone((a0, kw0))
        ex = _clone(extra)
        if "self_loop_grad_targets" in ex:
            vals, vec = ex["self_loop_grad_targets"]
            pre = [v.clone() for v in vals]
            ex["self_loop_grad_targets"] = (*vals, vec)
        kw.update(ex)
        res = pristine(*a, **kw)
        rec = {"extra": _clone(extra), "v_k": res[0].clone(),
               "aw": None if res[1] is None else [t.clone() for t in res[1:7]],
               "last_rel": (None if len(res) < 8 or res[7] is None else res[7].clone()),
               "has_last": len(res) == 8,
               "grad_col_post": None if kw.get("grad_col_log_probs") is None else kw["grad_col_log_probs"].clone()}
        if "self_loop_grad_targets" in ex:
            rec["targets_pre"] = pre
            rec["targets_post"] = [t.clone() for t in ex["self_loop_grad_targets"][:7]]
        out["cases"][name] = rec
        print(f"[{name}] W={W} S={S} active={int(mask.sum())} |v|={float(res[0].abs().max()):.3e}")
    torch.save(out, OUT)
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
