"""Full-size comparison with the reference's Triton path (configs 2 and 3) on the same GPU.

At full size neither fp32 result is exact: the reference adds its gradient columns in fp32 running
sums (per-wave ``_scatter_accum`` sums and per-element atomics), ours in fp64 per-CTA slots, and
the implicit gradients amplify rounding of the forward state.  So the comparison has three parts,
all on the same generated problem (``gen.generate(config, seed=1000*config)``):

1. forward intermediates (loss, E-step vectors, ``pibar_row_max``, every Pi / Pibar element):
   ours against the reference's, at the benchmark's tolerances;
2. backward of ONE forward state -- the reference's own intermediates, fed to every backward as
   the reference's ``bench/backward.py`` feeds golden ones -- by the reference (twice: its
   run-to-run spread), by our fused engine, by our call-by-call driver (the reference's glue
   structure: fp32 running sums) and by the same driver with fp64 totals
   (``exact_accumulation``); each against the EXACT backward of that state when the caller
   supplies one (the fp64 oracle on the host, affordable at config 2), else against the
   fp64-total driver;
3. both implementations' end-to-end results against the algorithm evaluated in float64
   (``tests/golden/fp64/config<N>.npz``, made by ``tests/golden/make_fp64.py``).

Errors are reported in units of the elementwise tolerance ``|d| / (atol + rtol |ref|)`` (1.0 = at
the tolerance) and as norm-wise relative errors.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent.parent
FP64 = ROOT / "tests" / "golden" / "fp64"
RTOL, ATOL, LOSS_RTOL = 1e-4, 1e-6, 1e-5
FWD_KEYS = ("E", "E_s1", "E_s2", "Ebar", "pibar_row_max", "pi_wave", "pibar_wave")
GRADS = ("grad_theta", "grad_col")


@torch.no_grad()
def compare(got, ref, rtol=RTOL, atol=ATOL) -> dict:
    """Elementwise tolerance units, max |d| and norm-wise relative error of ``got`` against
    ``ref`` (any shapes with the same number of elements; -inf positions must coincide)."""
    g = torch.as_tensor(got).detach().reshape(-1).double()
    r = torch.as_tensor(ref).detach().reshape(-1).to(g.device).double()
    ninf_g, ninf_r = torch.isneginf(g), torch.isneginf(r)
    mism = int((ninf_g != ninf_r).sum())
    fin = ~ninf_r & ~ninf_g
    d = (g[fin] - r[fin]).abs()
    rf = r[fin]
    units = float((d / (atol + rtol * rf.abs())).max()) if d.numel() else 0.0
    nrm = float(rf.norm())
    return {"tol_units": units if mism == 0 else float("inf"), "max_abs": float(d.max()) if d.numel() else 0.0,
            "norm_rel": float(d.norm()) / nrm if nrm > 0 else float(d.norm()), "ninf_mismatch": mism,
            "nan": int(torch.isnan(g).sum())}


def compare_grads(g, ref) -> dict:
    return {name: compare(a, b) for name, a, b in zip(GRADS, g, ref)}


def load_fp64(config: int, meta: dict) -> dict | None:
    """The float64 evaluation of ``config``'s problem, or None when it is absent or was made for a
    different problem (size counters or seed differ)."""
    path = FP64 / f"config{config}.npz"
    if not path.exists():
        return None
    z = dict(np.load(path))
    if int(z["S"]) != int(meta["S"]) or int(z["C"]) != int(meta["C"]) or int(z["seed"]) != int(meta["seed"]):
        return None
    return z


def timed(fn):
    """(result, ms) of ``fn()`` with CUDA events on the current stream."""
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    out = fn()
    b.record()
    torch.cuda.synchronize()
    return out, a.elapsed_time(b)


def reference_timing(ref_runtime, cap, device, steps: int) -> dict:
    """Median forward / backward ms of the reference's Triton path over ``steps`` solves after one
    warm-up solve (CUDA events; the warm-up includes Triton's JIT compilation)."""
    theta = cap["inputs"]["theta"].to(device)
    cw = cap["inputs"]["col_weights"].to(device)
    st = ref_runtime.make_static(cap, device)
    (_, sv), f0 = timed(lambda: ref_runtime.run_forward(st, theta, cw))
    _, b0 = timed(lambda: ref_runtime.run_backward(st, theta, cw, sv))
    del sv
    f_ms, b_ms = [], []
    for _ in range(steps):
        (_, sv), fm = timed(lambda: ref_runtime.run_forward(st, theta, cw))
        _, bm = timed(lambda: ref_runtime.run_backward(st, theta, cw, sv))
        f_ms.append(fm)
        b_ms.append(bm)
        del sv
    fwd, bwd = float(np.median(f_ms)), float(np.median(b_ms))
    return {"fwd_ms": fwd, "bwd_ms": bwd, "ms_per_solve": fwd + bwd, "solves_per_s": 1000.0 / (fwd + bwd),
            "first_solve_ms": f0 + b0, "steps": steps}


@torch.no_grad()
def full_size_parity(config: int, cap: dict, device, *, ref_runtime, our_runtime, glue=None,
                     exact_backward=None) -> dict:
    """Run the reference's Triton path and ours on ``cap`` and return the comparison report
    (see the module docstring).  ``glue`` (this project's ``kbench_b200.glue``) adds the
    call-by-call driver's backward, with fp32 running sums and with fp64 totals;
    ``exact_backward(saved_on_host) -> (grad_theta, grad_col)`` supplies the exact backward of a
    forward state."""
    theta = cap["inputs"]["theta"].to(device)
    cw = cap["inputs"]["col_weights"].to(device)
    rep: dict = {"config": config, "S": int(cap["meta"]["S"]), "C": int(cap["meta"]["C"])}

    st_r = ref_runtime.make_static(cap, device)
    loss_r, sv_r = ref_runtime.run_forward(st_r, theta, cw)
    g_r = ref_runtime.run_backward(st_r, theta, cw, sv_r)
    g_r2 = ref_runtime.run_backward(st_r, theta, cw, sv_r)
    _, sv_r2 = ref_runtime.run_forward(st_r, theta, cw)
    rep["ref_forward_repeat_bitwise"] = bool(all(torch.equal(sv_r[k], sv_r2[k]) for k in FWD_KEYS))
    del sv_r2

    st_o = our_runtime.make_static(cap, device)
    loss_o, sv_o = our_runtime.run_forward(st_o, theta, cw)
    g_o = our_runtime.run_backward(st_o, theta, cw, sv_o)
    rep["loss"] = {"ours": float(loss_o), "ref": float(loss_r),
                   "rel": abs(float(loss_o) - float(loss_r)) / abs(float(loss_r))}
    rep["forward_vs_ref"] = {k: compare(sv_o[k], sv_r[k]) for k in FWD_KEYS}

    # ---- backward of one forward state (the reference's) ----
    same = {"ref": g_r, "ref_repeat": g_r2, "engine": our_runtime.run_backward(st_o, theta, cw, sv_r)}
    # the engine's own run-to-run spread (its children's adjoint rows are added with fp32 atomics)
    rep["engine_repeat"] = compare_grads(our_runtime.run_backward(st_o, theta, cw, sv_r), same["engine"])
    if glue is not None:
        st_w = our_runtime.make_static(cap, device, engine="wrappers")
        same["wrappers"] = glue.implicit_grad(st_w, theta, cw, sv_r)
        same["wrappers_fp64_totals"] = glue.implicit_grad(st_w, theta, cw, sv_r, exact_accumulation=True)
    torch.cuda.synchronize()
    rep["same_state_vs_ref"] = {k: compare_grads(v, g_r) for k, v in same.items() if k != "ref"}
    if "wrappers_fp64_totals" in same:
        # the fused engine against the reference-structured driver with the engine's accumulation
        rep["engine_vs_fp64_totals"] = compare_grads(same["engine"], same["wrappers_fp64_totals"])
    if exact_backward is not None:
        host = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else v) for k, v in sv_r.items()}
        yard, yname = exact_backward(host), "fp64_oracle"
    else:
        yard, yname = same.get("wrappers_fp64_totals"), "wrappers_fp64_totals"
    rep["same_state_yardstick"] = yname if yard is not None else None
    if yard is not None:
        yard = tuple((y if torch.is_tensor(y) else torch.from_numpy(np.asarray(y))).to(device) for y in yard)
        rep["same_state_vs_yardstick"] = {k: compare_grads(v, yard) for k, v in same.items() if k != yname}

    # ---- end to end against the float64 evaluation ----
    z = load_fp64(config, cap["meta"])
    if z is not None:
        rows = torch.from_numpy(z["sample_rows"]).to(device)
        e2e = {}
        for name, loss, sv, g in (("ours", loss_o, sv_o, g_o), ("ref", loss_r, sv_r, g_r)):
            e2e[name] = {
                "loss_rel": abs(float(loss) - float(z["loss"])) / abs(float(z["loss"])),
                "E": compare(sv["E"], z["E"]), "pibar_row_max": compare(sv["pibar_row_max"], z["pibar_row_max"]),
                "pi_rows": compare(sv["pi_wave"][rows], z["pi_rows"]),
                "pibar_rows": compare(sv["pibar_wave"][rows], z["pibar_rows"]),
                **compare_grads(g, (torch.from_numpy(z["grad_theta"]), torch.from_numpy(z["grad_col"]))),
            }
        rep["end_to_end_vs_fp64"] = e2e
    else:
        rep["end_to_end_vs_fp64"] = None
    return rep
