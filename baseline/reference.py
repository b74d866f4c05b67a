"""The unmodified reference (SisyphusMountain/kernel-bench), installed under ``baseline/_ref``.

``baseline/_ref`` is git-ignored and travels with the repository snapshot to the GPU box.  It holds
the reference's Python package ``kbench`` (installed with pip from a copy of the checkout) and the
reference's ``bench/`` scripts (its correctness gate ``bench/check.py`` and the whole-pass and
per-kernel replays it drives), which are not part of the package.  Install once, in a container
that has the reference checkout::

    python baseline/reference.py --install <path-to-reference-checkout>

Two uses:

* :func:`stock_runtime` imports the reference's own ``kbench.runtime`` -- its frozen glue over its
  stock Triton kernels -- for timing the reference's Triton path on the same GPU and comparing
  results with it (``bench.py``, ``tests/test_gpu_reference_triton.py``);
* :func:`checkout_copy` lays out a scratch copy of the reference checkout (package + ``bench/``)
  whose kernel modules re-export this project's wrappers -- the drop-in recipe, applied to a
  copy -- so the reference's unchanged glue, runtime and ``bench/check.py`` run on the
  sm_100a kernels (``tests/test_gpu_reference_gate.py``).
"""

from __future__ import annotations

import argparse
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref"

# kbench/core/kernels/<module>.py -> the re-export that replaces it (the drop-in recipe)
SHIMS = {
    "wave_step": "from kbench_b200.kernels.wave_step import compute_wave_step, compute_leaf_initial_wave_step",
    "dts_fused": "from kbench_b200.kernels.dts_fused import compute_dts_forward",
    "e_step": ("from kbench_b200.kernels.e_step import e_fixed_point_triton, e_step_triton_autograd, "
               "_launch_e_step_forward_2d, _TritonEStep2D"),
    "wave_backward": ("from kbench_b200.kernels.wave_backward import active_mask_from_rhs_absmax_fused, "
                      "wave_backward_uniform_fused, dts_cross_backward_accum_fused, "
                      "uniform_cross_pibar_vjp_tree_from_ud_fused"),
    "wave_tangent": ("from kbench_b200.kernels.wave_tangent import compute_wave_step_tangent, "
                     "compute_wave_step_tangent_selfloop"),
    "dts_tangent": "from kbench_b200.kernels.dts_tangent import compute_dts_tangent",
    "e_step_tangent": "from kbench_b200.kernels.e_step_tangent import e_tangent_fixed_point, _launch_e_step_tangent_2d",
    "wave_so": "from kbench_b200.kernels.wave_so import wave_backward_so",
    "dts_so": "from kbench_b200.kernels.dts_so import dts_backward_so",
    "e_step_so": "from kbench_b200.kernels.e_step_so import e_step_backward_so",
}


def available() -> bool:
    """The reference package is installed."""
    return (REF / "kbench" / "runtime.py").exists()


def gate_available() -> bool:
    """The package and the reference's ``bench/`` scripts are installed."""
    return available() and (REF / "bench" / "check.py").exists()


def unavailable_reason() -> str | None:
    """Why the reference's Triton path cannot run here (None when it can)."""
    if not available():
        return "reference not installed in baseline/_ref (python baseline/reference.py --install <checkout>)"
    try:
        import triton  # noqa: F401
    except Exception as exc:  # noqa: BLE001
        return f"triton not importable: {exc}"
    import torch
    if not torch.cuda.is_available():
        return "no CUDA device"
    return None


def stock_runtime():
    """The reference's ``kbench.runtime`` over its stock Triton kernels (imported from
    ``baseline/_ref``).  A process that imports it must not also import a :func:`checkout_copy`."""
    if not available():
        raise RuntimeError(unavailable_reason())
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import kbench
    if Path(kbench.__file__).resolve().parent != (REF / "kbench").resolve():
        raise RuntimeError(f"another kbench package shadows the reference: {kbench.__file__}")
    from kbench import runtime
    return runtime


def checkout_copy(dst: Path, data: Path | None = None, *, shim: bool = True) -> Path:
    """Lay out ``dst`` as a reference checkout: ``dst/kbench`` (the installed package; with
    ``shim``, its ``core/kernels/<module>.py`` replaced by the re-exports of :data:`SHIMS`),
    ``dst/bench`` and, if given, ``dst/data`` (golden captures).  Run the reference's scripts from
    there with ``kernel-bench_b200`` on ``PYTHONPATH``.  ``shim=False`` keeps the stock Triton
    kernels (the control run of the same gate)."""
    if not gate_available():
        raise RuntimeError("reference package or bench/ scripts not installed in baseline/_ref")
    dst = Path(dst)
    shutil.copytree(REF / "kbench", dst / "kbench", ignore=shutil.ignore_patterns("__pycache__"))
    shutil.copytree(REF / "bench", dst / "bench", ignore=shutil.ignore_patterns("__pycache__"))
    kdir = dst / "kbench" / "core" / "kernels"
    for mod, line in (SHIMS.items() if shim else ()):
        (kdir / f"{mod}.py").write_text(
            f'"""Drop-in: this module re-exports the sm_100a implementation."""\n{line}  # noqa: F401\n')
    if data is not None:
        shutil.copytree(data, dst / "data")
    return dst


def install(checkout: Path) -> None:
    """pip-install the reference package into ``baseline/_ref`` (from a scratch copy: the build
    writes into its source tree) and copy its ``bench/`` scripts beside it."""
    checkout = Path(checkout).resolve()
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "kernel-bench"
        shutil.copytree(checkout, src, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                        "--find-links", "/opt/wheelhouse", "--target", str(REF), str(src)], check=True)
    if (REF / "bench").exists():
        shutil.rmtree(REF / "bench")
    shutil.copytree(checkout / "bench", REF / "bench", ignore=shutil.ignore_patterns("__pycache__"))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--install", type=Path, required=True, help="path of the reference checkout")
    install(ap.parse_args().install)
    print(f"installed into {REF}")
