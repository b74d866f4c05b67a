"""The CPU oracle against golden outputs of the reference itself (pristine Triton kernels run by
tests/golden/make_golden.py).  This pins the oracle that the GPU parity tests compare against."""

import numpy as np
import pytest

from _util import (OFF_DISTRIBUTION, assert_close, assert_forward_well_conditioned, assert_loss, golden_names,
                   load_golden, oracle_static)
from oracle import kb_oracle as O

NAMES = golden_names()
SAVED = ("pi_wave", "pibar_wave", "E", "E_s1", "E_s2", "Ebar", "log_pS", "log_pD", "log_pL", "max_coupling",
         "col_log_probs", "pibar_row_max")


def test_goldens_present():
    assert len(NAMES) >= 3


@pytest.mark.parametrize("name", NAMES)
def test_oracle_forward_matches_reference(name):
    cap, out = load_golden(name)
    loss, saved = O.forward(oracle_static(cap), cap["inputs"]["theta"], cap["inputs"]["col_weights"])
    assert_loss(loss, out["loss"])
    if name in OFF_DISTRIBUTION:
        assert_forward_well_conditioned(name, saved, out)
        return
    for k in ("pi_wave", "pibar_wave", "E", "Ebar", "pibar_row_max"):
        assert_close(k, saved[k], out[k])


@pytest.mark.parametrize("name", NAMES)
def test_oracle_backward_matches_reference(name):
    cap, out = load_golden(name)
    saved = {k: out[k] for k in SAVED}
    gt, gc = O.backward(oracle_static(cap), cap["inputs"]["theta"], cap["inputs"]["col_weights"], saved)
    assert_close("grad_theta", gt, out["grad_theta"])
    assert_close("grad_col", gc, out["grad_col"])


def test_planted_mistake_is_caught():
    """A deliberate error planted in the oracle's output must fail the comparison."""
    cap, out = load_golden(NAMES[0])
    loss, saved = O.forward(oracle_static(cap), cap["inputs"]["theta"], cap["inputs"]["col_weights"])
    bad = saved["pi_wave"].copy()
    bad[bad.shape[0] // 2, 3] += 0.01
    with pytest.raises(AssertionError):
        assert_close("pi_wave", bad, out["pi_wave"])


RELRES = [n for n in NAMES if "relres" in load_golden(n)[1]]


@pytest.mark.parametrize("name", RELRES)
def test_oracle_backward_relres_matches_reference(name):
    """The backward's convergence diagnostics (reference glue with ``collect_backward_relres``):
    per family the largest |last Neumann term| / |v| and the largest |v|."""
    cap, out = load_golden(name)
    saved = {k: out[k] for k in SAVED}
    rel: dict = {}
    O.backward_accumulators(oracle_static(cap), saved, relres=rel,
                            use_col_weights=not O.col_weights_are_uniform(cap["inputs"]["col_weights"]))
    assert_close("relres", rel["relres"], out["relres"])
    assert_close("vk_mag", rel["vk_mag"], out["vk_mag"])
