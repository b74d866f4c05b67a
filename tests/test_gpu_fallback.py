"""The fused forward's log-space recomputation, off the benchmark's rate distribution.

The engine iterates each row in linear space relative to a per-row scale; that is exact only
while nonzero values stay within 2^-100 of the row scale and the linear constants are >= 2^-26
(``kb_engine.cu``).  Two goldens made by the reference's pristine kernels leave that range:
``rowfallback_s63`` (loss rate x 2^5, transfer x 2^-10: rows spanning more than 100 binades, the
per-row recomputation) and ``forcelog_s31`` (transfer x 2^-30: constants below 2^-26, every row
recomputed).  Both schedules (dataflow and level launches) and both forward kernels (tour and
plain) must take the log-space path and match the reference's values where fp32 determines them
(the loss, every Pi element carrying at least 2^-20 of its row's largest value -- no -inf where
the reference has row mass --, the row maxima and the E-step vectors; ``tests/_util.py``
``OFF_DISTRIBUTION`` says why the Pibar denominators are not compared there)."""

import pytest
import torch

from _util import assert_forward_well_conditioned, assert_loss, load_golden

pytestmark = pytest.mark.gpu
VARIANTS = {"dataflow": {}, "levels": {"_flow": False}, "levels_plain": {"_flow": False, "_tour_forward": False}}


def _forward(name, variant, cuda):
    from kbench_b200 import gen, runtime
    cap, out = load_golden(name)
    capt = gen.to_torch(cap)
    static = runtime.make_static(capt, cuda)
    for k, v in VARIANTS[variant].items():
        setattr(static, k, v)
    theta = capt["inputs"]["theta"].to(cuda)
    cw = capt["inputs"]["col_weights"].to(cuda)
    loss, saved = runtime.run_forward(static, theta, cw)
    torch.cuda.synchronize()
    return cap, out, loss, saved, int(static._fallback_rows.item())


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_rows_beyond_linear_range_recomputed(variant, cuda):
    cap, out, loss, saved, n_fb = _forward("rowfallback_s63", variant, cuda)
    C = int(cap["meta"]["C"])
    assert 0 < n_fb < C, n_fb
    assert_loss(float(loss), out["loss"])
    assert_forward_well_conditioned("rowfallback_s63", {k: v.cpu().numpy() for k, v in saved.items() if torch.is_tensor(v)}, out)


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_constants_below_linear_range_force_log_space(variant, cuda):
    from kbench_b200 import engine
    cap, out, loss, saved, n_fb = _forward("forcelog_s31", variant, cuda)
    assert n_fb == int(cap["meta"]["C"]), n_fb
    assert_loss(float(loss), out["loss"])
    assert_forward_well_conditioned("forcelog_s31", {k: v.cpu().numpy() for k, v in saved.items() if torch.is_tensor(v)}, out)
    assert engine.LINEAR_MIN_LOG2 == -26.0
