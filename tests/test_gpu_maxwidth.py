"""Rows wider than the fused engine's 4,095 columns (up to the library maximum of 8,192): the
runtime routes them to the call-by-call driver, whose drop-in kernels must hold the whole row
on chip; checked against the oracle on a small family over an 8,191-column species tree."""

import pytest
import torch

from _util import assert_close, assert_loss
from kbench_b200 import engine, gen, runtime
from oracle import kb_oracle as O

pytestmark = pytest.mark.gpu


def test_widest_rows_run_on_the_wrapper_driver(cuda):
    cfg = gen.ProblemConfig("wide8191", 4096, 12, 2, 3, 0,
                            solver_options={"e_tol": 1e-6, "e_max_iter": 50, "pi_iters": 6, "neumann_terms": 4})
    cap = gen.generate(cfg, seed=8191, as_torch=False)
    st = dict(cap["static"])
    st["solver_options"] = cap["meta"]["solver_options"]
    loss_ref, saved_ref = O.forward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"])
    gt_ref, gc_ref = O.backward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"], saved_ref)
    static = runtime.make_static(gen.to_torch(cap), cuda)
    assert int(static.state_helpers["S"]) == 8191 and not engine.supported(static)
    theta = torch.from_numpy(cap["inputs"]["theta"]).to(cuda)
    col = torch.from_numpy(cap["inputs"]["col_weights"]).to(cuda)
    loss, saved = runtime.run_forward(static, theta, col)
    assert_loss(float(loss), loss_ref)
    for k in ("pi_wave", "pibar_wave", "pibar_row_max", "E"):
        assert_close(k, saved[k].cpu().numpy(), saved_ref[k])
    gt, gc = runtime.run_backward(static, theta, col, saved)
    assert_close("grad_theta", gt.cpu().numpy(), gt_ref)
    assert_close("grad_col", gc.cpu().numpy(), gc_ref)
