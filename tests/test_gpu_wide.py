"""Parity at the benchmark's row widths (S = 511 and S = 4095, the configs' species trees) and two
odd widths (S = 79, S = 599) on small gene families, so the CPU oracle finishes in seconds: the fused engine (forward tour kernel
and the packed-table kernel it replaces, backward level kernel) against the oracle, with the
production solver settings (pi_iters = 16, neumann_terms = 16)."""

import numpy as np
import pytest
import torch

from _util import assert_close, assert_loss
from kbench_b200 import gen, runtime, tree
from oracle import kb_oracle as O

pytestmark = pytest.mark.gpu

CASES = {
    "S511": gen.ProblemConfig("wide511", 256, 24, 3, 8, 0, solver_options=dict(gen.CONFIGS[2].solver_options)),
    "S4095": gen.ProblemConfig("wide4095", 2048, 32, 3, 10, 0, solver_options=dict(gen.CONFIGS[3].solver_options)),
    # widths whose padded row is not a multiple of 128 columns (NTV = 96 and 608): the backward
    # runs them one column per thread so that its block stays whole warps
    "S79": gen.ProblemConfig("wide79", 40, 24, 3, 8, 0, solver_options=dict(gen.CONFIGS[1].solver_options)),
    "S599": gen.ProblemConfig("wide599", 300, 24, 3, 8, 0, solver_options=dict(gen.CONFIGS[2].solver_options)),
}
_REF = {}


def _reference(name):
    if name not in _REF:
        cap = gen.generate(CASES[name], seed=4242, as_torch=False)
        st = dict(cap["static"])
        st["solver_options"] = cap["meta"]["solver_options"]
        loss, saved = O.forward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"])
        gt, gc = O.backward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"], saved)
        _REF[name] = (cap, loss, saved, gt, gc)
    return _REF[name]


@pytest.mark.parametrize("tour", [True, False])
@pytest.mark.parametrize("name", sorted(CASES))
def test_engine_forward_backward_vs_oracle(cuda, name, tour):
    cap, loss_ref, saved_ref, gt_ref, gc_ref = _reference(name)
    S = int(cap["meta"]["S"])
    assert tree.tour_layout(S) is not None
    static = runtime.make_static(gen.to_torch(cap), cuda)
    static._tour_forward = tour
    theta = torch.from_numpy(cap["inputs"]["theta"]).to(cuda)
    col = torch.from_numpy(cap["inputs"]["col_weights"]).to(cuda)
    loss, saved = runtime.run_forward(static, theta, col)
    assert int(static._fallback_rows.item()) == 0
    assert_loss(float(loss), loss_ref)
    for k in ("pi_wave", "pibar_wave", "pibar_row_max", "E", "Ebar"):
        assert_close(k, saved[k].cpu().numpy(), saved_ref[k])
    gt, gc = runtime.run_backward(static, theta, col, saved)
    assert_close("grad_theta", gt.cpu().numpy(), gt_ref)
    assert_close("grad_col", gc.cpu().numpy(), gc_ref)
