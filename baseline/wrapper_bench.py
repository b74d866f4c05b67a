"""Per-wrapper timing of one forward + backward pass driven by the reference's own glue.

Run as a script in a process whose ``kbench`` is either the reference's stock package
(``baseline/_ref``: its Triton kernels) or a checkout copy whose kernel modules re-export this
project's wrappers (``reference.checkout_copy``).  The glue's kernel entry points -- the names it
binds at import time, the same targets as the reference's ``capture/capture.py`` -- are wrapped
with CUDA-event timers; one warm-up pass (Triton's JIT, caches), then one timed pass of
``runtime.run_forward`` + ``run_backward`` on a generated problem.  Prints one JSON object:
per wrapper the number of calls and the summed milliseconds between its start and end events on
the current stream (host-side synchronisation inside a wrapper, such as the reference E-step's
per-iteration ``.item()``, is part of its time), plus the whole pass.

    python baseline/wrapper_bench.py --root <checkout> --config 2
"""

from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

# (glue module, attribute): the call sites the reference's capture tool patches, plus the E-step
# fixed point and the active mask
TARGETS = [
    ("kbench.core.inference.forward", "compute_leaf_initial_wave_step"),
    ("kbench.core.inference.forward", "compute_wave_step"),
    ("kbench.core.inference.forward", "compute_dts_forward"),
    ("kbench.core.inference.solver", "e_fixed_point_triton"),
    ("kbench.api._implicit_grad", "active_mask_from_rhs_absmax_fused"),
    ("kbench.api._implicit_grad", "compute_dts_forward"),
    ("kbench.api._implicit_grad", "wave_backward_uniform_fused"),
    ("kbench.api._implicit_grad", "dts_cross_backward_accum_fused"),
    ("kbench.api._implicit_grad", "uniform_cross_pibar_vjp_tree_from_ud_fused"),
    ("kbench.api._implicit_grad", "e_step_triton_autograd"),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--root", type=Path, required=True, help="checkout whose kbench package is used")
    ap.add_argument("--config", type=int, default=2)
    args = ap.parse_args()
    sys.path.insert(0, str(args.root))
    sys.path.insert(1, str(ROOT / "kernel-bench_b200"))
    import torch
    from kbench import runtime
    from kbench_b200 import gen

    records: dict = {}
    active = [False]

    def wrap(mod, attr):
        fn = getattr(mod, attr)
        key = f"{mod.__name__.rsplit('.', 1)[-1]}.{attr}"

        def timed(*a, **k):
            if not active[0]:
                return fn(*a, **k)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*a, **k)
            e1.record()
            records.setdefault(key, []).append((e0, e1))
            return out

        setattr(mod, attr, timed)

    for mp, attr in TARGETS:
        wrap(importlib.import_module(mp), attr)
    cap = gen.generate(args.config, seed=1000 * args.config)
    dev = torch.device("cuda:0")
    st = runtime.make_static(cap, dev)
    theta, cw = cap["inputs"]["theta"].to(dev), cap["inputs"]["col_weights"].to(dev)

    def one_pass():
        loss, saved = runtime.run_forward(st, theta, cw)
        runtime.run_backward(st, theta, cw, saved)
        return loss

    one_pass()
    torch.cuda.synchronize()
    active[0] = True
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    loss = one_pass()
    p1.record()
    torch.cuda.synchronize()
    out = {"kbench": str(Path(importlib.import_module("kbench").__file__).parent), "config": args.config,
           "loss": float(loss), "pass_ms": p0.elapsed_time(p1),
           "wrappers": {k: {"calls": len(v), "ms": round(sum(a.elapsed_time(b) for a, b in v), 3)}
                        for k, v in sorted(records.items())}}
    print("WRAPPER_BENCH " + json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
