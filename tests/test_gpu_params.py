"""The column-weight normaliser kernels (``kb_col_normalizer`` / ``kb_col_normalizer_vjp``)
against a plain PyTorch fp32 statement of reference ``extract_parameters.py:41-65`` (the round
loop of gathers), forward and VJP, on the species trees of the benchmark's configs."""

import math

import pytest
import torch

from _util import assert_close
from kbench_b200 import gen, params, runtime

pytestmark = pytest.mark.gpu


def _loop_normalizer(clp, parent, depth):
    """Reference ``extract_parameters.py:41-65`` restated with torch ops (test reference only)."""
    S = int(clp.numel())
    probs = torch.exp2(clp)
    parent = parent.to(device=clp.device, dtype=torch.long)
    cur = torch.arange(S, device=clp.device, dtype=torch.long)
    mass = torch.zeros((S,), device=clp.device, dtype=clp.dtype)
    zero = mass.new_zeros(())
    for _ in range(max(1, int(depth))):
        valid = (cur >= 0) & (cur < S)
        safe = cur.clamp(0, max(S - 1, 0))
        mass = mass + torch.where(valid, probs.index_select(0, safe), zero)
        cur = torch.where(valid, parent.index_select(0, safe), torch.full_like(cur, -1))
    vm = 1.0 - mass
    return torch.where(vm > 0.0, -torch.log2(vm.clamp_min(torch.finfo(clp.dtype).tiny)),
                       clp.new_full((S,), float("-inf")))


@pytest.mark.parametrize("cfg", [1, 2, 3, 4])
@pytest.mark.parametrize("peaked", [False, True])
def test_normalizer_matches_loop(cfg, peaked, cuda):
    cap = gen.generate(gen.ProblemConfig(f"norm{cfg}", gen.CONFIGS[cfg].n_species, 8, 2, 4, 0), seed=11 + cfg)
    static = runtime.make_static(cap, cuda)
    sh = static.state_helpers
    S = int(sh["S"])
    g = torch.Generator(device="cpu").manual_seed(cfg)
    w = torch.randn(S, generator=g) * (8.0 if peaked else 1.0)
    if peaked:  # push some root paths' mass close to 1 (the cancellation and -inf branches)
        w[int(torch.argmax(w))] += 30.0
    w = w.to(cuda).requires_grad_(True)
    w2 = w.detach().clone().requires_grad_(True)
    clp = params.col_log_probs_from_weights(w)
    clp2 = params.col_log_probs_from_weights(w2)
    out = params.col_valid_log_normalizer(clp, sh["node_parent"], int(sh["max_ancestor_depth"]),
                                          node_child1=sh["node_child1"], node_child2=sh["node_child2"])
    ref = _loop_normalizer(clp2, sh["node_parent"], int(sh["max_ancestor_depth"]))
    # same summation order and the same exp2/log2: equal to the last bit
    assert torch.equal(out.detach().isneginf(), ref.detach().isneginf())
    fin = ~ref.detach().isneginf()
    assert torch.equal(out.detach()[fin], ref.detach()[fin])
    cot = torch.randn(S, generator=g).to(cuda)
    (gw,) = torch.autograd.grad((out.masked_fill(~fin, 0.0) * cot).sum(), w)
    (gw2,) = torch.autograd.grad((ref.masked_fill(~fin, 0.0) * cot).sum(), w2)
    # the per-ancestor sums run in another order (subtree sums vs scattered adds) and may cancel:
    # elementwise rel 1e-5 plus an absolute floor of 1e-6 of the largest entry
    ref_g = gw2.cpu().numpy()
    assert_close("grad_col_weights", gw.cpu().numpy(), ref_g, rtol=1e-5, atol=1e-6 * float(abs(ref_g).max()))
    assert math.isfinite(float(gw.abs().sum()))
