"""The dataflow backward's deterministic form (the default; ``static._deterministic_backward``): every
split writes its two children's contributions to edge rows (zeros from an inactive row), and a row
adds its seed and its incoming edge rows in edge order when it starts -- no atomics, so the solved
adjoint rows are bitwise the same on every run, whatever order the rows ran in.  Checked on the medium config (8k rows,
up to dozens of parents per row): two runs give bitwise equal adjoint rows and gradients equal to
fp64 association (the per-row column sums meet in fp64 per-CTA slots), and the result agrees with
the atomic form (the edge rows switched off) within the gradient tolerance."""

import pytest
import torch

from _util import assert_close, assert_close_rows
from kbench_b200 import engine, gen, runtime

pytestmark = pytest.mark.gpu


def _backward(static, theta, col, saved, C, S, dev):
    v = torch.zeros((C, S), device=dev, dtype=torch.float32)
    gt, gc = engine.backward(static, theta, col, saved, v_out=v)
    torch.cuda.synchronize()
    return v, gt, gc


def test_backward_adjoint_rows_are_run_to_run_identical(cuda):
    cap = gen.generate(2, seed=2000)
    static = runtime.make_static(cap, cuda)
    theta = cap["inputs"]["theta"].to(cuda)
    col = cap["inputs"]["col_weights"].to(cuda)
    _, saved = runtime.run_forward(static, theta, col)
    C, S = (int(x) for x in saved["pi_wave"].shape)
    static._deterministic_backward = True
    v0, gt0, gc0 = _backward(static, theta, col, saved, C, S, cuda)
    assert getattr(static, "_edge_scratch", None) is not None, "the deterministic form did not run"
    v1, gt1, gc1 = _backward(static, theta, col, saved, C, S, cuda)
    assert torch.equal(v0, v1)
    # the column sums: each row's own fp32 sums go to fp64 per-CTA slots, whose row groups vary run
    # to run -- fp64 association only, far below one fp32 ulp of the gradients
    assert_close("grad_theta (repeat)", gt1.cpu().numpy(), gt0.cpu().numpy(), rtol=2.5e-7, atol=1e-12)
    assert_close("grad_col (repeat)", gc1.cpu().numpy(), gc0.cpu().numpy(), rtol=2.5e-7, atol=1e-12)
    static._deterministic_backward = False
    va, gta, gca = _backward(static, theta, col, saved, C, S, cuda)
    assert_close_rows("adjoint rows vs atomic form", va.cpu().numpy(), v0.cpu().numpy())
    assert_close("grad_theta vs atomic form", gta.cpu().numpy(), gt0.cpu().numpy())
    assert_close("grad_col vs atomic form", gca.cpu().numpy(), gc0.cpu().numpy())
