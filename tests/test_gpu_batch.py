"""Family batches on the GPU: the fused engine chunk by chunk (fp64 accumulators shared by the
chunks, one E adjoint) against the oracle over the whole batch, and against the engine run on one
static holding every family."""

import numpy as np
import pytest
import torch

from _batch_ranks import SEED, TINY, oracle_static
from _util import assert_close, assert_loss
from kbench_b200 import batch, gen, runtime
from oracle import kb_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("chunk", [1, 4])
def test_engine_batch_matches_oracle_and_whole_static(cuda, chunk):
    cap = gen.generate(TINY, seed=SEED, as_torch=False)
    st = oracle_static(cap)
    loss_ref, saved = O.forward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"])
    gt_ref, gc_ref = O.backward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"], saved)

    chunks = batch.build_chunks(TINY, 0, TINY.n_families, chunk, seed=SEED, workers=1)
    fb = batch.FamilyBatch(chunks, TINY.n_families, batch.EngineSolver(cuda))
    theta = torch.from_numpy(cap["inputs"]["theta"]).to(cuda)
    col = torch.from_numpy(cap["inputs"]["col_weights"]).to(cuda)
    res = fb.step(theta, col)
    assert_loss(float(res.loss), loss_ref)
    assert_close("grad_theta", res.grad_theta.cpu().numpy(), gt_ref)
    assert_close("grad_col", res.grad_col.cpu().numpy(), gc_ref)

    static = runtime.make_static(gen.to_torch(cap), cuda)
    loss_w, saved_w = runtime.run_forward(static, theta, col)
    gt_w, gc_w = runtime.run_backward(static, theta, col, saved_w)
    assert_loss(float(res.loss), float(loss_w))
    assert_close("grad_theta (whole static)", res.grad_theta.cpu().numpy(), gt_w.cpu().numpy())
    assert_close("grad_col (whole static)", res.grad_col.cpu().numpy(), gc_w.cpu().numpy())
