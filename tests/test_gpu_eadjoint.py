"""The one-launch E adjoint (``kb_e_adjoint_solve``) against the general path it replaces for a
shared E row: the BiCGSTAB of ``glue.bicgstab`` over one E-step VJP launch per matvec and the
parameter VJP through autograd (reference ``_implicit_grad.py:28-94, 373-475``).  Both run on the
same saved forward state; the solution ``w`` and the gradients must agree to the parity
tolerance (rel 1e-4, abs 1e-6).  The non-converged path raises the reference's error."""

import pytest
import torch

from _util import assert_close, golden_names, load_golden
from kbench_b200 import gen, glue, runtime

pytestmark = pytest.mark.gpu

WIDE = {
    "S511": gen.ProblemConfig("wide511", 256, 24, 3, 8, 0, solver_options=dict(gen.CONFIGS[2].solver_options)),
    "S4095": gen.ProblemConfig("wide4095", 2048, 32, 3, 10, 0, solver_options=dict(gen.CONFIGS[3].solver_options)),
}


def _both_paths(capt, cuda):
    static = runtime.make_static(capt, cuda)
    theta = capt["inputs"]["theta"].to(cuda)
    cw = capt["inputs"]["col_weights"].to(cuda)
    loss, saved = runtime.run_forward(static, theta, cw)
    if saved["E"].shape[0] != 1:
        pytest.skip("E is per item: the general path applies")
    out = {}
    for dev in (True, False):
        glue.DEVICE_E_ADJOINT = dev
        try:
            gt, gc = runtime.run_backward(static, theta, cw, saved)
        finally:
            glue.DEVICE_E_ADJOINT = True
        torch.cuda.synchronize()
        out[dev] = (static._last_e_adjoint.reshape(-1).cpu().numpy(), gt.cpu().numpy(), gc.cpu().numpy())
    return out


def _check(out):
    (w1, gt1, gc1), (w0, gt0, gc0) = out[True], out[False]
    assert_close("w", w1, w0)
    assert_close("grad_theta", gt1, gt0)
    assert_close("grad_col", gc1, gc0)


@pytest.mark.parametrize("name", golden_names())
def test_one_launch_matches_general_path_golden(name, cuda):
    cap, _ = load_golden(name)
    _check(_both_paths(gen.to_torch(cap), cuda))


@pytest.mark.parametrize("name", sorted(WIDE))
def test_one_launch_matches_general_path_wide(name, cuda):
    cap = gen.generate(WIDE[name], seed=4242)
    _check(_both_paths(cap, cuda))


def test_not_converged_raises_and_device_stays_usable(cuda):
    from kbench_b200.kernels.e_step import e_adjoint_solve
    cap = gen.generate(WIDE["S511"], seed=4242)
    static = runtime.make_static(cap, cuda)
    theta = cap["inputs"]["theta"].to(cuda)
    cw = cap["inputs"]["col_weights"].to(cuda)
    _, saved = runtime.run_forward(static, theta, cw)
    sh = static.state_helpers
    S = int(sh["S"])
    gen_ = torch.Generator(device="cpu").manual_seed(5)
    g = [torch.randn(1, S, generator=gen_).to(cuda) for _ in range(4)]
    args = (saved["E"], saved["log_pS"], saved["log_pD"], saved["log_pL"], saved["max_coupling"],
            saved["col_log_probs"], sh["node_parent"], sh["node_child1"], sh["node_child2"],
            int(sh["max_ancestor_depth"]), *g)
    with pytest.raises(RuntimeError, match="failed after 1 iterations"):
        e_adjoint_solve(*args, n_fam=3, max_iter=1, tol=1e-30)
    w, gp = e_adjoint_solve(*args, n_fam=3, max_iter=500, tol=1e-7)
    assert bool(torch.isfinite(w).all()) and bool(torch.isfinite(gp).all())
    assert e_adjoint_solve.last_iters >= 1
