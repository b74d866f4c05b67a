"""Failure detection of the dataflow schedule, without a GPU fault: a dependency count that is one
too high leaves a row that is never released; every wait on it must give up after its poll bound,
the launch must end with the error flag set (the engine raises: at the end of the forward, or of
the backward that follows when the forward's check is deferred), and the device must stay usable
(a normal forward right after matches the level schedule bitwise)."""

import pytest
import torch

from kbench_b200 import engine, gen, runtime

pytestmark = pytest.mark.gpu


def test_unreleased_row_times_out_and_reports(cuda, monkeypatch):
    cap = gen.generate(1, seed=1000)
    static = runtime.make_static(cap, cuda)
    theta = cap["inputs"]["theta"].to(cuda)
    col = cap["inputs"]["col_weights"].to(cuda)
    plan = engine.build_plan(static)
    root = int(cap["static"]["wave_layout"]["root_row_ids"][0])
    good = plan.dep0.clone()
    plan.dep0[root] += 1  # the root waits for a child that does not exist
    monkeypatch.setattr(engine, "FLOW_MAX_POLLS", 2000)
    with pytest.raises(RuntimeError, match="dataflow wait gave up"):
        runtime.run_forward(static, theta, col)
    # a caller that defers the forward's check to the backward that follows gets it there
    with pytest.raises(RuntimeError, match="dataflow wait gave up"):
        _, saved = runtime.run_forward(static, theta, col, check_errors=False)
        runtime.run_backward(static, theta, col, saved)
    plan.dep0.copy_(good)
    monkeypatch.setattr(engine, "FLOW_MAX_POLLS", 1 << 25)
    loss_f, saved_f = runtime.run_forward(static, theta, col)
    static._flow = False
    loss_l, saved_l = runtime.run_forward(static, theta, col)
    torch.cuda.synchronize()
    assert torch.equal(saved_f["pi_wave"], saved_l["pi_wave"])
    assert float(loss_f) == float(loss_l)
