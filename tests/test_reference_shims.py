"""Host-side check of the drop-in recipe: in a copy of the reference checkout whose kernel modules
re-export this project's wrappers, the reference's frozen glue binds OUR functions (by name, at
import time: ``kbench/core/inference/forward.py:3-4``, ``solver.py:7``, ``api/_implicit_grad.py:4-16``)
and nothing on that path imports Triton.  Runs on the CPU; the GPU run of the same layout is
``test_gpu_reference_gate.py``."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
from baseline import reference  # noqa: E402

PROBE = r"""
import sys
sys.path.insert(0, sys.argv[1])
import kbench.runtime
import kbench.core.inference.forward as fw
import kbench.core.inference.solver as so
import kbench.api._implicit_grad as ig
import kbench.core.kernels.e_step as es
bound = {
    "compute_wave_step": fw.compute_wave_step, "compute_leaf_initial_wave_step": fw.compute_leaf_initial_wave_step,
    "compute_dts_forward": fw.compute_dts_forward, "e_fixed_point_triton": so.e_fixed_point_triton,
    "ig.compute_dts_forward": ig.compute_dts_forward, "e_step_triton_autograd": ig.e_step_triton_autograd,
    "wave_backward_uniform_fused": ig.wave_backward_uniform_fused,
    "dts_cross_backward_accum_fused": ig.dts_cross_backward_accum_fused,
    "uniform_cross_pibar_vjp_tree_from_ud_fused": ig.uniform_cross_pibar_vjp_tree_from_ud_fused,
    "active_mask_from_rhs_absmax_fused": ig.active_mask_from_rhs_absmax_fused,
    "_launch_e_step_forward_2d": es._launch_e_step_forward_2d,
}
for name, fn in bound.items():
    print(name, fn.__module__)
print("triton_loaded", "triton" in sys.modules)
print("kbench_from", kbench.runtime.__file__)
"""


@pytest.mark.skipif(not reference.gate_available(), reason="reference not installed in baseline/_ref")
def test_shimmed_glue_binds_b200_wrappers(tmp_path):
    root = reference.checkout_copy(tmp_path / "kernel-bench")
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT / "kernel-bench_b200")
    res = subprocess.run([sys.executable, "-c", PROBE, str(root)], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr
    lines = dict(line.split(" ", 1) for line in res.stdout.strip().splitlines())
    assert lines.pop("triton_loaded") == "False"
    assert Path(lines.pop("kbench_from")).resolve().is_relative_to(root.resolve())
    for name, mod in lines.items():
        assert mod.startswith("kbench_b200.kernels."), (name, mod)
