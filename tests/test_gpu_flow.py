"""The dataflow schedule (one persistent launch, rows start when their dependencies are done)
against the level-by-level schedule on the medium config (8k rows, 51 dependency levels): the
forward must be bitwise identical (same per-row arithmetic, only the start times differ); the
backward's column sums are added in a different order (fp64 totals), so the gradients agree to
the stated tolerance."""

import pytest
import torch

from _util import assert_close, assert_loss
from kbench_b200 import gen, runtime

pytestmark = pytest.mark.gpu


def test_flow_matches_level_schedule(cuda):
    cap = gen.generate(2, seed=2000)
    static = runtime.make_static(cap, cuda)
    theta = cap["inputs"]["theta"].to(cuda)
    col = cap["inputs"]["col_weights"].to(cuda)
    out = {}
    for flow in (False, True):
        static._flow = flow
        loss, saved = runtime.run_forward(static, theta, col)
        gt, gc = runtime.run_backward(static, theta, col, saved)
        out[flow] = (float(loss), saved, gt, gc)
    (l0, s0, gt0, gc0), (l1, s1, gt1, gc1) = out[False], out[True]
    for k in ("pi_wave", "pibar_wave", "pibar_row_max"):
        assert torch.equal(s0[k], s1[k]), k
    n_leaf = int(cap["static"]["wave_layout"]["wave_metas"][0]["W"])  # leaf rows store no split reduction
    assert torch.equal(s0["dts_wave"][n_leaf:], s1["dts_wave"][n_leaf:])
    assert_loss(l1, l0)
    assert_close("grad_theta", gt1.cpu().numpy(), gt0.cpu().numpy())
    assert_close("grad_col", gc1.cpu().numpy(), gc0.cpu().numpy())

