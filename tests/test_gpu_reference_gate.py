"""The reference's own correctness gate, unchanged, on this project's kernels.

A scratch copy of the reference checkout is laid out whose ``kbench/core/kernels/*.py`` re-export
this project's wrappers (the drop-in recipe of INTEGRATION.md), with golden captures made by the
reference's own ``capture/capture.py`` from its pristine kernels (``tests/golden/make_capture.py``:
a config-1 problem with 19 per-wrapper snapshots, the adjoint-options problem and a
weighted-column problem).  Then the reference's ``bench/check.py`` runs as shipped:

* FORWARD: ``kbench.runtime.run_forward`` -- the frozen glue (``solve_e_pi``, ``pi_wave_forward``)
  calling our wrappers wave by wave -- against the golden ``loss, pi_wave, E, pibar_row_max``;
* BACKWARD: ``run_backward`` (``implicit_grad_loglik_vjp_wave``, fed the golden forward
  intermediates) against the golden ``grad_theta, grad_col``;
* KERNELS: every captured wrapper call rebuilt with its storage aliasing and replayed on our
  wrapper, every tensor argument, keyword and return compared after the call -- the in-place
  ``Pi_out`` / ``Pibar`` / ``accumulated_rhs`` / ``pibar_ud`` states, the ``aw*`` buckets, ``v_k``,
  the parameter gradients -- at the positions the capture marked meaningful.

Its rule: a tensor passes when its largest absolute OR largest relative disagreement is within
the tolerance (``bench/_common.py:80-120``).  Run at the gate's default 2e-3 and at the benchmark's
1e-4 / 1e-6.  Needs the reference installed in ``baseline/_ref`` (package and ``bench/``); skipped
without it.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CAPTURES = ROOT / "tests" / "golden" / "capture"

sys.path.insert(0, str(ROOT))
from baseline import reference  # noqa: E402


def run_check(tmp_path, *extra, shim=True):
    """Run the reference's ``bench/check.py`` in a scratch checkout; returns (rc, output)."""
    if not reference.gate_available():
        pytest.skip("reference package / bench scripts not installed in baseline/_ref")
    root = reference.checkout_copy(tmp_path / "kernel-bench", data=CAPTURES, shim=shim)
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT / "kernel-bench_b200")
    res = subprocess.run([sys.executable, str(root / "bench" / "check.py"), *extra], cwd=root, env=env,
                         capture_output=True, text=True, timeout=900)
    out = res.stdout + res.stderr
    print(out)
    return res.returncode, out


@pytest.mark.gpu
def test_reference_check_gate(cuda, tmp_path):
    """``bench/check.py`` at its own default tolerance."""
    rc, out = run_check(tmp_path)
    assert rc == 0 and "ALL PASS" in out
    # every captured wrapper call was replayed
    assert out.count("\n--- ") == 19


@pytest.mark.gpu
def test_reference_check_gate_tight(cuda, tmp_path):
    """The same gate at the benchmark's tolerances (rel 1e-4, abs 1e-6)."""
    rc, out = run_check(tmp_path, "--rtol", "1e-4", "--atol", "1e-6")
    assert rc == 0 and "ALL PASS" in out
