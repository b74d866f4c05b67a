"""Entry points: ``make_static`` / ``run_forward`` / ``run_backward``.

Same contract as the reference's ``kbench/runtime.py:29-115`` (``FORWARD_SAVED_NAMES``, the
``static`` namespace, theta -> (loss, saved), saved -> (grad_theta, grad_col)).  Two drivers:

* ``engine="fused"`` (default): the B200 engine of ``engine.py`` (dependency-level schedule,
  fused all-iteration wave sweeps, fused per-row adjoint);
* ``engine="wrappers"``: the reference-structured driver of ``glue.py`` that calls the drop-in
  wrappers one iteration at a time, as the reference's frozen glue does.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import torch

from .options import SolverOptions

FORWARD_SAVED_NAMES = (
    "E", "E_s1", "E_s2", "Ebar", "root_rows", "pi_wave", "pibar_wave",
    "pibar_row_max", "log_pS", "log_pD", "log_pL", "max_coupling", "col_log_probs",
)


def move_to_device(obj, device):
    if isinstance(obj, np.ndarray):
        obj = torch.from_numpy(np.ascontiguousarray(obj))
    if torch.is_tensor(obj):
        return obj.to(device)
    if isinstance(obj, dict):
        return {k: move_to_device(v, device) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(move_to_device(v, device) for v in obj)
    return obj


def make_static(captured: dict, device, *, engine: str = "fused") -> SimpleNamespace:
    st = captured["static"]
    so = SolverOptions(**captured["meta"]["solver_options"])
    so.validate()
    if engine not in ("fused", "wrappers"):
        raise ValueError("engine must be 'fused' or 'wrappers'")
    static = SimpleNamespace(
        wave_layout=move_to_device(st["wave_layout"], device),
        state_helpers=move_to_device(st["state_helpers"], device),
        rate_item_idx=move_to_device(st["rate_item_idx"], device),
        itemwise=bool(st["itemwise"]),
        statewise=bool(st["statewise"]),
        solver_options=so,
        warm_E=None,
        engine=engine,
        # flat row-ordered split arrays of a device-built layout (kbench_b200.builder), else None
        flat_layout=move_to_device(st.get("flat_layout"), device),
    )
    sh = static.state_helpers
    for key in ("S", "max_ancestor_depth"):
        if torch.is_tensor(sh[key]):
            sh[key] = int(sh[key])
    for meta in static.wave_layout["wave_metas"]:
        for key in ("start", "W", "n_eq1", "ge2_max_fanout"):
            if key in meta and torch.is_tensor(meta[key]):
                meta[key] = int(meta[key])
    return static


def run_forward(static, theta, col_weights, *, check_errors=True):
    """theta -> (loss, dict of forward intermediates).

    The fused engine also returns ``saved["dts_wave"]`` (the per-row split reductions), which its
    backward reuses instead of recomputing them; every other key is the reference's.
    ``check_errors=False`` (a caller that runs ``run_backward`` next) leaves the engine's dataflow
    error check to the end of that backward, so the host does not wait for the forward."""
    from .glue import nll_from_root_rows
    extras = {}
    with torch.no_grad():
        if getattr(static, "engine", "fused") == "fused":
            from . import engine
            out, extras = engine.forward(static, theta, col_weights, check_errors=check_errors)
        else:
            from . import glue
            out = glue.solve_e_pi(static, theta, col_weights)
        loss = nll_from_root_rows(out[4], out[0])
    saved = dict(zip(FORWARD_SAVED_NAMES, out))
    saved.update(extras)
    return loss, saved


def run_backward(static, theta, col_weights, saved: dict, *, check_errors=True):
    """(forward intermediates) -> (grad_theta, grad_col).  ``check_errors=False`` (a solver loop
    that calls :func:`check_errors` itself, e.g. once after the loop) skips the engine's dataflow
    error check, the one host synchronisation of a solve."""
    if getattr(static, "engine", "fused") == "fused":
        from . import engine
        return engine.backward(static, theta, col_weights, saved, check_errors=check_errors)
    from . import glue
    return glue.implicit_grad(static, theta, col_weights, saved)


def check_errors(static) -> None:
    """Raise if a dataflow launch of the fused engine on ``static`` gave up a wait since the last
    check (see ``run_forward`` / ``run_backward``'s ``check_errors``); one host synchronisation."""
    if getattr(static, "engine", "fused") == "fused":
        from . import engine
        engine.check_flow_errors(static)
