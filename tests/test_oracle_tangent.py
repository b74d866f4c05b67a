"""The CPU tangent oracle against the reference's own forward-mode tangent (``jvp_root_scores``
with the fused fixed-count self-loop) run by tests/golden/make_golden.py --tangent."""

import numpy as np
import pytest

from _util import GOLDEN, assert_close, assert_close_rows, load_golden, oracle_static
from oracle import kb_oracle_tangent as OT

NAMES = sorted(p.stem for p in (GOLDEN / "tangent").glob("*.npz"))


def load_tangent(name):
    return dict(np.load(GOLDEN / "tangent" / f"{name}.npz"))


def test_tangent_goldens_present():
    assert len(NAMES) >= 1


@pytest.mark.parametrize("name", NAMES)
def test_oracle_tangent_matches_reference(name):
    cap, out = load_golden(name)
    tg = load_tangent(name)
    st = oracle_static(cap)
    k = 0
    while f"v{k}" in tg:
        roots, dpi, dpibar, dc = OT.jvp_root_scores(st, cap["inputs"]["theta"], tg[f"v{k}"], out,
                                                   self_iters=int(tg["self_iters"]))
        for key in ("dE", "dE_s1", "dE_s2", "dEbar", "dlog_pS", "dlog_pD", "dlog_pL", "dmax_coupling"):
            assert_close(f"{key}[{k}]", dc["raw"][key], tg[f"{key}{k}"])
        assert_close_rows(f"dPi[{k}]", dpi, tg[f"dPi{k}"])
        assert_close_rows(f"dPibar[{k}]", dpibar, tg[f"dPibar{k}"])
        assert_close_rows(f"roots[{k}]", roots, tg[f"roots{k}"])
        k += 1
    assert k >= 1
