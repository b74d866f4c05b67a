"""Produce the reference's own golden captures (``data/<label>/whole.pt`` and per-wrapper
``kernels/*.pt`` snapshots) for generated problems, so that the reference's unchanged gate
``bench/check.py`` -- whole forward, whole backward and the per-kernel replay -- can be run on this
project's kernels (``tests/test_gpu_reference_gate.py``).

Runs ONLY in a container with the reference checkout (``--reference``).  It:
  1. swaps the reference's *pristine* kernels (``experiments/pristine_kernels/*``, its golden
     producer, ``capture/capture.py:1-19``) in for ``kbench.core.kernels.*`` exactly as
     ``make_golden.py`` does, and runs them on the CPU under ``TRITON_INTERPRET=1``;
  2. writes the generated problem as the fixture the capture tool reads (``fixtures/<label>.pt``,
     the ``captured`` dict: meta, static, inputs) into a scratch folder;
  3. runs the reference's own ``capture/capture.py`` ``capture_size`` (imported from the checkout,
     not copied) with its ``FIXTURES`` / ``DATA`` folders pointed at the scratch folder and
     ``tests/golden/capture/``.  That records ``whole.pt`` (inputs, forward intermediates, loss
     and gradients) and, for the first label, pre/post snapshots of up to 4 distinct calls of each
     of the 7 kernel wrappers with the run-twice noise floors and don't-care masks
     (``capture/capture.py:164-210``).

One harness-side adjustment: ``measure_noise`` rebuilds each call with
``rebuild(pre_ref, pool, device=DEVICE)`` (``kbench/_capture_io.py:70-91``), which relies on the
move to the device copying the pool tensors.  On the CPU ``.to("cpu")`` returns the pool tensor
itself, so the two noise runs would add their in-place updates (``accumulated_rhs``, the
parameter gradients, ``grad_col_log_probs``, ``pibar_ud``) into the stored pre-states, and the
replay could not reproduce the golden post-states even with the pristine kernels.  Here the
capture module's ``rebuild`` hands out fresh copies instead (one per aliasing group, so aliasing is
kept), which is what the reference's GPU capture gets from the device move.  With it, the
pristine kernels reproduce every snapshot on replay.  (The interpreter runs atomics in order, so
the recorded noise floors are zero: the replay gate is the strict 2e-3 one.)

Usage:  python tests/golden/make_capture.py --reference <path-to-reference-checkout>
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import make_golden  # noqa: E402  (sets up the package path; install_pristine)
from kbench_b200 import gen  # noqa: E402

OUT = HERE / "capture"

# label: (config or ProblemConfig, seed, solver option overrides, per-wrapper kernel snapshots)
CASES = {
    "cfg1_s1000": (1, 1000, {}, True),
    "options_s63": (1, 6363, {"use_adjoint_pruning": False, "pibar_side_threshold": 1e-3}, False),
    "weighted_s31": (gen.ProblemConfig("weighted", 16, 20, 4, 10, 0), 3131, {"_col_weights_seed": 77}, False),
}


def build_case(cfg, seed, overrides):
    overrides = dict(overrides)
    cw_seed = overrides.pop("_col_weights_seed", None)
    cap = gen.generate(cfg, seed=seed, solver_options=overrides)
    if cw_seed is not None:
        S = int(cap["meta"]["S"])
        w = np.random.Generator(np.random.PCG64(cw_seed)).standard_normal(S).astype(np.float32)
        cap["inputs"]["col_weights"] = torch.from_numpy(w)
    return cap


def fresh_rebuild(rebuild):
    """``rebuild`` whose tensors are copies of the pool entries (one per aliasing group)."""

    def wrapped(ref_struct, pool, *, device=None):
        memo = {}

        def conv(o):
            if torch.is_tensor(o):
                if id(o) not in memo:
                    memo[id(o)] = o.detach().clone()
                return memo[id(o)]
            if isinstance(o, dict):
                return {k: conv(v) for k, v in o.items()}
            if isinstance(o, (list, tuple)):
                return type(o)(conv(v) for v in o)
            return o

        return conv(rebuild(ref_struct, pool, device=None))

    return wrapped


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--cases", default=",".join(CASES))
    args = ap.parse_args()
    torch.set_num_threads(1)
    ref = args.reference.resolve()
    make_golden.install_pristine(ref)
    capture = make_golden._load_module("kb_reference_capture", ref / "capture" / "capture.py")
    capture.DEVICE = "cpu"
    capture.rebuild = fresh_rebuild(capture.rebuild)
    OUT.mkdir(exist_ok=True)
    capture.DATA = OUT
    with tempfile.TemporaryDirectory() as tmp:
        capture.FIXTURES = Path(tmp)
        for label in args.cases.split(","):
            cfg, seed, ov, kernels = CASES[label]
            cap = build_case(cfg, seed, ov)
            torch.save(cap, Path(tmp) / f"{label}.pt")
            capture.capture_size(label, capture_kernels=kernels, per_wrapper=4)


if __name__ == "__main__":
    main()
