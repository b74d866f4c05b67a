"""Forward-mode tangent (the tangent config) on the GPU.

* the reference-structured driver (drop-in wrappers) against the reference's own tangent
  (golden fixtures), at the reference's saved forward state;
* the fused multi-direction engine (``jvp_batch``) against that driver on the same state;
* the tangent against central finite differences of the fused forward (the benchmark's
  acceptance check, rel 1e-3 in norm) on a problem with the S = 511 species tree.
"""

import numpy as np
import pytest
import torch

from _util import GOLDEN, assert_close, assert_close_rows, load_golden
from kbench_b200 import gen, runtime, tangent

pytestmark = pytest.mark.gpu

NAMES = sorted(p.stem for p in (GOLDEN / "tangent").glob("*.npz"))
SAVED = ("E", "E_s1", "E_s2", "Ebar", "pi_wave", "pibar_wave", "pibar_row_max", "log_pS", "log_pD", "log_pL",
         "max_coupling", "col_log_probs")


def _static(cap, dev):
    return runtime.make_static(gen.to_torch(cap), dev)


@pytest.mark.parametrize("name", NAMES)
def test_wrapper_tangent_matches_reference(cuda, name):
    cap, out = load_golden(name)
    tg = dict(np.load(GOLDEN / "tangent" / f"{name}.npz"))
    static = _static(cap, cuda)
    sv = {k: torch.from_numpy(np.asarray(out[k])).to(cuda) for k in SAVED}
    theta = torch.from_numpy(cap["inputs"]["theta"]).to(cuda)
    k = 0
    while f"v{k}" in tg:
        v = torch.from_numpy(tg[f"v{k}"]).to(cuda)
        roots, full = tangent.jvp_root_scores(static, theta, v, sv, self_iters=int(tg["self_iters"]),
                                              return_full=True)
        for key in ("dE", "dE_s1", "dE_s2", "dEbar", "dlog_pS", "dlog_pD", "dlog_pL", "dmax_coupling"):
            assert_close(f"{key}[{k}]", full[key].reshape(-1).cpu().numpy(), tg[f"{key}{k}"])
        assert_close_rows(f"dPi[{k}]", full["dPi"].cpu().numpy(), tg[f"dPi{k}"])
        assert_close_rows(f"dPibar[{k}]", full["dPibar"].cpu().numpy(), tg[f"dPibar{k}"])
        assert_close_rows(f"roots[{k}]", roots.cpu().numpy(), tg[f"roots{k}"])
        k += 1


@pytest.mark.parametrize("name", NAMES)
def test_fused_batch_tangent_matches_wrapper_driver(cuda, name):
    cap, _ = load_golden(name)
    tg = dict(np.load(GOLDEN / "tangent" / f"{name}.npz"))
    static = _static(cap, cuda)
    theta = torch.from_numpy(cap["inputs"]["theta"]).to(cuda)
    col = torch.from_numpy(cap["inputs"]["col_weights"]).to(cuda)
    _, saved = runtime.run_forward(static, theta, col)
    V = torch.stack([torch.from_numpy(tg[f"v{k}"]) for k in range(2)]).to(cuda)
    it = int(tg["self_iters"])
    roots_b, full_b = tangent.jvp_batch(static, theta, V, saved, self_iters=it, return_full=True)
    for k in range(2):
        roots, full = tangent.jvp_root_scores(static, theta, V[k], saved, self_iters=it, return_full=True)
        assert_close(f"dE[{k}]", full_b["dE"][k].cpu().numpy(), full["dE"].reshape(-1).cpu().numpy())
        assert_close_rows(f"dPi[{k}]", full_b["dPi"][k].cpu().numpy(), full["dPi"].cpu().numpy())
        assert_close_rows(f"dPibar[{k}]", full_b["dPibar"][k].cpu().numpy(), full["dPibar"].cpu().numpy())
        assert_close_rows(f"roots[{k}]", roots_b[k].cpu().numpy(), roots.cpu().numpy())


def fd_check(static, theta, col, V, roots, eps):
    """Norm-wise relative error of the tangent against central differences of the forward."""
    errs = []
    for k in range(V.shape[0]):
        lp, sp = runtime.run_forward(static, theta + eps * V[k], col)
        lm, sm = runtime.run_forward(static, theta - eps * V[k], col)
        fd = (sp["root_rows"].double() - sm["root_rows"].double()) / (2 * eps)
        t = roots[k].double()
        fin = torch.isfinite(fd) & torch.isfinite(t)
        errs.append(float((fd[fin] - t[fin]).norm() / fd[fin].norm()))
    return errs


def test_tangent_matches_finite_differences(cuda):
    cfg = gen.ProblemConfig("fd511", 256, 48, 4, 12, 0,
                            solver_options=dict(gen.CONFIGS[2].solver_options, e_tol=1e-9))
    cap = gen.generate(cfg, seed=5151)
    static = runtime.make_static(cap, cuda)
    theta = cap["inputs"]["theta"].to(cuda)
    col = cap["inputs"]["col_weights"].to(cuda)
    _, saved = runtime.run_forward(static, theta, col)
    g = torch.Generator().manual_seed(5000)
    V = torch.randn((2, theta.shape[0], 3), generator=g).to(cuda)
    roots = tangent.jvp_batch(static, theta, V, saved)
    errs = fd_check(static, theta, col, V, roots, eps=1e-2)
    assert max(errs) < 1e-3, errs
