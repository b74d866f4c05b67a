"""The CPU exact-Hessian HVP oracle against the reference's own ``newton/hvp_exact.py``
``make_exact_hvp`` run by tests/golden/make_golden.py --hvp (its second-order kernels under
``TRITON_INTERPRET=1``), and the symmetry a Hessian-vector product must have.  The compared
vectors are signed accumulations over every wave: ``assert_close_vec`` (rel 1e-4 of the vector's
scale per element, and norm-wise)."""

import numpy as np
import pytest

from _util import GOLDEN, assert_close_vec, load_golden, oracle_static
from oracle import kb_oracle_hvp as OH

NAMES = sorted(p.stem for p in (GOLDEN / "hvp").glob("*.npz"))
DEBUG = ("d_gE", "d_gpD", "d_gpS", "d_gmc", "d_gEbar", "d_gEs1", "d_gEs2", "dq_E", "dwE")


def load_hvp(name):
    return dict(np.load(GOLDEN / "hvp" / f"{name}.npz"))


def _case(name):
    cap, out = load_golden(name)
    saved = {k: np.asarray(v) for k, v in out.items() if k not in ("loss", "grad_theta", "grad_col")}
    return cap, oracle_static(cap), saved


def test_hvp_goldens_present():
    assert len(NAMES) >= 1


@pytest.mark.parametrize("name", NAMES)
def test_oracle_hvp_matches_reference(name):
    cap, st, saved = _case(name)
    hv = load_hvp(name)
    theta, cw = cap["inputs"]["theta"], cap["inputs"]["col_weights"]
    cache = OH.point_cache(st, theta, cw, saved)
    k = 0
    while f"u{k}" in hv:
        dbg: dict = {}
        hu = OH.hvp(st, theta, cw, saved, hv[f"u{k}"], cache=cache, debug_out=dbg)
        for key in DEBUG:
            assert_close_vec(f"{key}[{k}]", dbg[key].reshape(-1), hv[f"{key}{k}"])
        assert_close_vec(f"Hu[{k}]", hu, hv[f"hu{k}"])
        k += 1
    assert k >= 1


@pytest.mark.parametrize("name", NAMES)
def test_oracle_hvp_is_symmetric(name):
    """u1 . (H u0) = u0 . (H u1) up to the truncations of the solves (Neumann terms, self-loop
    iterations): the relative asymmetry stays small."""
    cap, st, saved = _case(name)
    theta, cw = cap["inputs"]["theta"], cap["inputs"]["col_weights"]
    S = theta.shape[0]
    rng = np.random.default_rng(9)
    u0, u1 = (rng.standard_normal(3 * S).astype(np.float32) for _ in range(2))
    cache = OH.point_cache(st, theta, cw, saved)
    h0 = OH.hvp(st, theta, cw, saved, u0, cache=cache).astype(np.float64)
    h1 = OH.hvp(st, theta, cw, saved, u1, cache=cache).astype(np.float64)
    a, b = float(u1 @ h0), float(u0 @ h1)
    scale = np.linalg.norm(h0) * np.linalg.norm(u1) + np.linalg.norm(h1) * np.linalg.norm(u0)
    assert abs(a - b) <= 1e-4 * scale, (a, b, scale)


def test_head_second_order_term_matches_finite_differences():
    """The closed-form smooth-head Hessian (the GPU driver uses the same formula) against central
    differences of the extraction's VJP at fixed cotangents."""
    from oracle import kb_oracle as O
    cap, st, _ = _case(NAMES[0])
    tree = O.Tree(st["state_helpers"])
    S = tree.S
    rng = np.random.default_rng(3)
    theta = rng.standard_normal((S, 3))
    u = rng.standard_normal((S, 3))
    cot = [rng.standard_normal(S).astype(np.float32) for _ in range(4)]
    cw = np.zeros(S, np.float32)
    eps = 1e-3

    def jt(th):
        g, _ = O.extract_parameters_vjp(th, cw, tree, *cot, np.zeros(S, np.float32), uniform_fast=True)
        return g.astype(np.float64)

    fd = (jt(theta + eps * u) - jt(theta - eps * u)) / (2 * eps)
    h = OH.head_hvp(theta, u, cot)
    assert np.abs(h - fd).max() <= 1e-3 * max(np.abs(fd).max(), 1e-6)
