"""GPU parity: the sm_100a path (both drivers) against the reference's golden outputs and the
CPU oracle, through the public runtime API and the drop-in wrappers."""

import numpy as np
import pytest
import torch

from _util import OFF_DISTRIBUTION, assert_close, assert_forward_well_conditioned, assert_loss, golden_names, load_golden

pytestmark = pytest.mark.gpu
NAMES = golden_names()


def _run(name, engine, cuda):
    from kbench_b200 import gen, runtime
    cap, out = load_golden(name)
    capt = gen.to_torch(cap)
    static = runtime.make_static(capt, cuda, engine=engine)
    theta = capt["inputs"]["theta"].to(cuda)
    cw = capt["inputs"]["col_weights"].to(cuda)
    loss, saved = runtime.run_forward(static, theta, cw)
    gsaved = {k: torch.as_tensor(out[k]).to(cuda) for k in runtime.FORWARD_SAVED_NAMES if k in out}
    gsaved["root_rows"] = gsaved["pi_wave"][static.wave_layout["root_row_ids"]]
    gt, gc = runtime.run_backward(static, theta, cw, gsaved)
    torch.cuda.synchronize()
    return out, loss, saved, gt, gc


@pytest.mark.parametrize("engine", ["wrappers", "fused"])
@pytest.mark.parametrize("name", NAMES)
def test_forward_backward_vs_reference_golden(name, engine, cuda):
    out, loss, saved, gt, gc = _run(name, engine, cuda)
    assert_loss(float(loss), out["loss"])
    if name in OFF_DISTRIBUTION:
        assert_forward_well_conditioned(name, {k: v.cpu().numpy() for k, v in saved.items() if torch.is_tensor(v)}, out)
    else:
        for k in ("pi_wave", "pibar_wave", "E", "Ebar", "pibar_row_max", "E_s1", "E_s2"):
            assert_close(k, saved[k].cpu().numpy(), out[k])
    assert_close("grad_theta", gt.cpu().numpy(), out["grad_theta"])
    assert_close("grad_col", gc.cpu().numpy(), out["grad_col"])


RELRES = [n for n in NAMES if "relres" in load_golden(n)[1]]


@pytest.mark.parametrize("name", RELRES)
def test_backward_relres_vs_reference_golden(name, cuda):
    """``return_last_increment`` through the call-by-call driver's ``collect_backward_relres``
    (the reference glue's diagnostics mode) against the reference's values."""
    from kbench_b200 import gen, glue, runtime
    cap, out = load_golden(name)
    capt = gen.to_torch(cap)
    static = runtime.make_static(capt, cuda, engine="wrappers")
    theta = capt["inputs"]["theta"].to(cuda)
    cw = capt["inputs"]["col_weights"].to(cuda)
    gsaved = {k: torch.as_tensor(out[k]).to(cuda) for k in runtime.FORWARD_SAVED_NAMES if k in out}
    gsaved["root_rows"] = gsaved["pi_wave"][static.wave_layout["root_row_ids"]]
    relres, vk_mag = glue.implicit_grad(static, theta, cw, gsaved, collect_backward_relres=True)
    assert_close("relres", relres.cpu().numpy(), out["relres"])
    assert_close("vk_mag", vk_mag.cpu().numpy(), out["vk_mag"])
