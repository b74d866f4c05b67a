"""Forward-mode tangent (JVP) of the root scores: ``d(Pi_root)/dtheta . v`` (the tangent config).

Two drivers, as for the primal solve:

* :func:`jvp_root_scores` -- the reference's ``newton/forward_tangent.py:105-215`` call sequence
  (parameter tangent, E tangent fixed point, then per size-wave the split tangent and the
  self-loop tangent), one direction, driving the drop-in wrappers of ``kbench_b200.kernels``;
* :func:`jvp_batch` -- the B200 engine: D directions at once, the E tangents of all directions in
  one launch and ONE launch per dependency level (``kb_level_tangent``: every (row, direction)
  pair of the level computes its split tangent and all ``self_iters`` self-loop steps on chip),
  reusing the primal split reductions the fused forward saved.

Both evaluate every Jacobian at the frozen primal state in ``saved`` (the forward's outputs) and,
with ``self_iters`` set, run the fixed-count Jacobi self-loop from a zero tangent (the reference's
fused path, matching the primal's ``pi_iters`` truncation).
"""

from __future__ import annotations

import math

import torch

from . import _lib, engine, tree
from .kernels._common import f32, i32, i64
from .kernels.dts_fused import compute_dts_forward
from .kernels.dts_tangent import compute_dts_tangent, parent_csr
from .kernels.e_step_tangent import e_tangent_fixed_point
from .kernels.wave_tangent import compute_wave_step_tangent, compute_wave_step_tangent_selfloop
from .params import as_item_param, as_item_state

_LN2 = math.log(2.0)


def _default_tol(dtype):
    """``forward_tangent.py:64-65``."""
    return 1e-12 if dtype == torch.float64 else 1e-6


def param_jvp_uniform(static, theta, v):
    """``forward_tangent.py:29-40``: tangent of ``extract_parameters_uniform`` along ``v``
    ([S,3] or a batch [D,S,3]).  With logits ``[0, theta]`` and ``p`` their base-2 softmax,
    ``d log2softmax_j = dl_j - sum_k p_k dl_k`` (``unnorm_row_max`` is a constant).  Returns
    (dlog_pS, dlog_pD, dlog_pL, dmax_coupling), each shaped like ``v[..., 0]``."""
    if not (static.statewise and not static.itemwise):
        raise ValueError("param_jvp_uniform: statewise, not itemwise layouts only")
    th = theta.detach()
    logits = torch.cat([th.new_zeros((*th.shape[:-1], 1)), th], dim=-1)
    p = torch.softmax(logits * _LN2, dim=-1)
    dl = torch.cat([v.new_zeros((*v.shape[:-1], 1)), v.to(th.dtype)], dim=-1)
    dr = dl - (p * dl).sum(dim=-1, keepdim=True)
    return dr[..., 0], dr[..., 1], dr[..., 2], dr[..., 3]


def _base_constants(sv, S):
    """``forward_tangent.py:43-61`` ``wave_step_constants``."""
    rows = int(sv["E"].shape[0])
    e = as_item_state(sv["E"], S, rows)
    return {
        "dl": 1.0 + as_item_state(sv["log_pD"], S, rows) + e, "ebar": as_item_state(sv["Ebar"], S, rows), "e": e,
        "sl1": as_item_state(sv["log_pS"], S, rows) + as_item_state(sv["E_s2"], S, rows),
        "sl2": as_item_state(sv["log_pS"], S, rows) + as_item_state(sv["E_s1"], S, rows),
        "mc": as_item_state(sv["max_coupling"].squeeze(-1), S, rows), "leaf": as_item_state(sv["log_pS"], S, rows),
        "pd_param": as_item_param(sv["log_pD"], rows, S), "ps_param": as_item_param(sv["log_pS"], rows, S),
    }


def tangent_constants(static, theta, v, sv, S, e_tol, raw_out=None):
    """``forward_tangent.py:68-100`` ``_wave_tangent_constants`` (one direction)."""
    dpS, dpD, dpL, dmc = param_jvp_uniform(static, theta, v)
    sh = static.state_helpers
    dE, dE_s1, dE_s2, dEbar = e_tangent_fixed_point(
        sv["E"], dpS, dpD, dpL, dmc, sv["log_pS"], sv["log_pD"], sv["log_pL"], sv["max_coupling"],
        sv["col_log_probs"], sh["node_parent"], sh["node_child1"], sh["node_child2"], int(sh["max_ancestor_depth"]),
        max_iter=int(static.solver_options.e_max_iter), tol=e_tol, use_col_weights=False)
    if raw_out is not None:
        raw_out.update(dlog_pS=dpS, dlog_pD=dpD, dlog_pL=dpL, dmax_coupling=dmc, dE=dE, dE_s1=dE_s1, dE_s2=dE_s2,
                       dEbar=dEbar)
    rows = int(sv["E"].shape[0])
    st = lambda t: as_item_state(t, S, rows)  # noqa: E731
    return {
        "dDL": st(dpD) + st(dE), "dEbar": st(dEbar), "dE": st(dE), "dSL1": st(dpS) + st(dE_s2),
        "dSL2": st(dpS) + st(dE_s1), "dMC": st(dmc), "dleaf": st(dpS),
        "dpd_param": as_item_param(dpD, rows, S), "dps_param": as_item_param(dpS, rows, S),
    }


@torch.no_grad()
def tangent_wave_cache(static, sv) -> dict:
    """The direction-independent part of :func:`jvp_root_scores`' wave loop, for callers that run
    many tangents at one point (the exact-Hessian HVP): per wave with splits, the primal split
    reduction ``dts_r`` and the split CSR of the tangent reduction (keyed by the wave's start row)."""
    sh, wl = static.state_helpers, static.wave_layout
    S = int(sh["S"])
    base = _base_constants(sv, S)
    out = {}
    for meta in wl["wave_metas"]:
        if "sl" not in meta:
            continue
        ws, W = int(meta["start"]), int(meta["W"])
        dts_r = compute_dts_forward(sv["pi_wave"], sv["pibar_wave"], meta["sl"], meta["sr"], sh["node_child1"],
                                    sh["node_child2"], W, meta["reduce_idx"], base["pd_param"], base["ps_param"],
                                    item_idx=static.rate_item_idx, log_split_probs=meta.get("log_split_probs"),
                                    n_eq1=meta.get("n_eq1"), eq1_reduce_idx=meta.get("eq1_reduce_idx"),
                                    ge2_ptr=meta.get("ge2_ptr"), ge2_parent_ids=meta.get("ge2_parent_ids"),
                                    ge2_max_fanout=meta.get("ge2_max_fanout"), item_offset=ws)
        out[ws] = {"dts_r": dts_r, "csr": parent_csr(meta["reduce_idx"], W)}
    return out


@torch.no_grad()
def jvp_root_scores(static, theta, v, sv, *, self_tol=None, self_max_iter=200, e_tol=None, self_iters=None,
                    return_full=False, wave_cache=None):
    """``forward_tangent.py:105-215`` driven through the drop-in wrappers (one direction):
    returns ``d(Pi_root)/dtheta . v`` [n_roots, S] (and, with ``return_full``, a dict with
    ``dPi``, ``dPibar``, the tangent constants and the raw parameter / E tangents).

    ``self_iters`` runs the fused fixed-count self-loop (the tangent config's setting); ``None``
    iterates each wave's self-loop to ``self_tol`` as the reference's adaptive path does.
    ``wave_cache``: :func:`tangent_wave_cache` at the same point (skips recomputing the primal
    split reductions)."""
    sh, wl = static.state_helpers, static.wave_layout
    S = int(sh["S"])
    if self_tol is None:
        self_tol = _default_tol(theta.dtype)
    if e_tol is None:
        e_tol = _default_tol(theta.dtype)
    item_idx = static.rate_item_idx
    leaf_state_idx = wl["leaf_state_index"].to(torch.int32)
    c1, c2, parent = sh["node_child1"], sh["node_child2"], sh["node_parent"]
    mad = int(sh["max_ancestor_depth"])
    base = _base_constants(sv, S)
    raw = {} if return_full else None
    dc = tangent_constants(static, theta, v, sv, S, e_tol, raw_out=raw)
    pi, pibar = sv["pi_wave"], sv["pibar_wave"]
    C = int(pi.shape[0])
    dpi = torch.zeros((C, S), device=pi.device, dtype=pi.dtype)
    dpibar = torch.zeros((C, S), device=pi.device, dtype=pi.dtype)
    consts = (base["mc"], dc["dMC"], base["dl"], dc["dDL"], base["ebar"], dc["dEbar"], base["e"], dc["dE"],
              base["sl1"], dc["dSL1"], base["sl2"], dc["dSL2"])

    def step(dts_r, d_dts, ws, W, has_leaf, store):
        compute_wave_step_tangent(pi, dpi, dpi, ws, W, S, *consts, sv["col_log_probs"], c1, c2, parent, mad, dts_r,
                                  d_dts, leaf_state_idx=leaf_state_idx, leaf_logp=base["leaf"],
                                  dleaf_logp=dc["dleaf"], item_idx=item_idx,
                                  dPibar_out=(dpibar if store else None), has_leaf_term=has_leaf,
                                  use_col_weights=False)

    for meta in wl["wave_metas"]:
        ws, W = int(meta["start"]), int(meta["W"])
        has_splits = "sl" in meta
        if has_splits:
            kw = dict(log_split_probs=meta.get("log_split_probs"), n_eq1=meta.get("n_eq1"),
                      eq1_reduce_idx=meta.get("eq1_reduce_idx"), ge2_ptr=meta.get("ge2_ptr"),
                      ge2_parent_ids=meta.get("ge2_parent_ids"), ge2_max_fanout=meta.get("ge2_max_fanout"),
                      item_offset=ws)
            wc = None if wave_cache is None else wave_cache[ws]
            if wc is None:
                dts_r = compute_dts_forward(pi, pibar, meta["sl"], meta["sr"], c1, c2, W, meta["reduce_idx"],
                                            base["pd_param"], base["ps_param"], item_idx=item_idx, **kw)
            else:
                dts_r = wc["dts_r"]
            d_dts = compute_dts_tangent(pi, pibar, dpi, dpibar, meta["sl"], meta["sr"], c1, c2, W,
                                        meta["reduce_idx"], base["pd_param"], base["ps_param"], dc["dpd_param"],
                                        dc["dps_param"], dts_r, item_idx, csr=None if wc is None else wc["csr"],
                                        **kw)
        else:
            dts_r = d_dts = None
        if self_iters is not None:
            compute_wave_step_tangent_selfloop(pi, dpi, ws, W, S, max(int(self_iters), 1), *consts,
                                               sv["col_log_probs"], c1, c2, parent, mad, dts_r, d_dts,
                                               leaf_state_idx=leaf_state_idx, leaf_logp=base["leaf"],
                                               dleaf_logp=dc["dleaf"], item_idx=item_idx, dPibar_out=dpibar,
                                               has_leaf_term=not has_splits, use_col_weights=False)
        else:
            prev = dpi.narrow(0, ws, W).clone()
            for _ in range(int(self_max_iter)):
                step(dts_r, d_dts, ws, W, not has_splits, store=False)
                cur = dpi.narrow(0, ws, W)
                diff = float((cur - prev).abs().max())
                scale = float(cur.abs().max())
                if diff <= self_tol * max(1.0, scale):
                    break
                prev = cur.clone()
            step(dts_r, d_dts, ws, W, not has_splits, store=True)
    roots = dpi.index_select(0, wl["root_row_ids"])
    if return_full:
        return roots, dict(dPi=dpi, dPibar=dpibar, dcst=dc, **raw)
    return roots


@torch.no_grad()
def jvp_batch(static, theta, V, saved, *, self_iters=None, e_tol=None, return_full=False):
    """Fused engine tangent for D directions ``V`` [D,S,3] at once: returns the root tangents
    [D, n_roots, S] (and, with ``return_full``, ``dPi`` / ``dPibar`` [D,C,S] plus the E and
    parameter tangents [D,S]).  ``saved`` must come from the fused forward (it carries the split
    reductions ``dts_wave``); ``self_iters`` defaults to the solver's ``pi_iters``."""
    so = static.solver_options
    sh, wl = static.state_helpers, static.wave_layout
    S = int(sh["S"])
    if "dts_wave" not in saved:
        raise ValueError("jvp_batch needs the fused forward's saved split reductions (saved['dts_wave'])")
    if tree.tour_layout(S) is None:
        raise ValueError(f"jvp_batch supports S <= 4095 (got {S})")
    if not engine.supported(static):
        raise ValueError("jvp_batch needs the fused engine's layout (statewise, shared theta)")
    V = V.reshape(-1, S, 3) if V.ndim == 2 else V
    D = int(V.shape[0])
    Pi, Pibar, dts = f32(saved["pi_wave"]), f32(saved["pibar_wave"]), f32(saved["dts_wave"])
    C = int(Pi.shape[0])
    dev = Pi.device
    G = int(saved["E"].shape[0])
    if G != 1:
        raise ValueError("jvp_batch supports one shared item row")
    e_tol = _default_tol(theta.dtype) if e_tol is None else e_tol
    st = _lib.stream_handle(dev)
    topo = engine._topo(static)
    tt = topo.tt
    plan = engine.build_plan(static)

    # parameter tangents [D,S] and the E tangents of all directions (one persistent CTA each)
    dpS, dpD, dpL, dmc = (f32(t.reshape(D, S)) for t in param_jvp_uniform(static, theta, V))
    E = f32(saved["E"])
    pS, pD, pL, mc = (f32(as_item_state(saved[k].squeeze(-1) if k == "max_coupling" else saved[k], S, 1))
                      for k in ("log_pS", "log_pD", "log_pL", "max_coupling"))
    dE, scratch, dE_s1, dE_s2, dEbar = (torch.empty((D, S), device=dev, dtype=torch.float32) for _ in range(5))
    iters = torch.zeros((D,), device=dev, dtype=torch.int32)
    _lib.call("kb_e_tangent_fixed_point", E.data_ptr(), dpS.data_ptr(), dpD.data_ptr(), dpL.data_ptr(),
              dmc.data_ptr(), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), mc.data_ptr(),
              f32(saved["col_log_probs"].reshape(-1)).data_ptr(), 0, tt.child1.data_ptr(), tt.child2.data_ptr(),
              tt.jumps.data_ptr(), tt.K, 1, S, D, int(so.e_max_iter), float(e_tol), None, dE.data_ptr(),
              scratch.data_ptr(), dE_s1.data_ptr(), dE_s2.data_ptr(), dEbar.data_ptr(), iters.data_ptr(), st)
    # tangent constants [D,S] (forward_tangent.py:89-100)
    dDL = (dpD + dE).contiguous()
    dSL1 = (dpS + dE_s2).contiguous()
    dSL2 = (dpS + dE_s1).contiguous()
    base = _base_constants({k: saved[k] for k in ("E", "Ebar", "E_s1", "E_s2", "log_pS", "log_pD",
                                                  "max_coupling")}, S)
    k = {n: f32(base[n]) for n in ("mc", "dl", "ebar", "e", "sl1", "sl2", "leaf")}
    pDp, pSp = f32(base["pd_param"]), f32(base["ps_param"])
    prs = 0 if int(pDp.shape[0]) == 1 else S
    dPi = torch.empty((D, C, S), device=dev, dtype=torch.float32)
    dPibar = torch.empty((D, C, S), device=dev, dtype=torch.float32)
    n_it = max(int(so.pi_iters if self_iters is None else self_iters), 1)
    leaf_state = i32(wl["leaf_state_index"])
    item_idx = i64(static.rate_item_idx)
    rows_ptr, sp_ptr = plan.rows.data_ptr(), plan.split_ptr.data_ptr()
    if getattr(static, "_flow", True) and getattr(static, "_tangent_pairs", True) and D % 2 == 0:
        n_items = C * (D // 2)
        queue = torch.empty((n_items,), device=dev, dtype=torch.int32)
        remaining = torch.empty((n_items,), device=dev, dtype=torch.int32)
        counters = torch.zeros((3,), device=dev, dtype=torch.int32)
        engine._launch(static, "kb_flow_tangent", 0, C, plan.row_split_ptr.data_ptr(), plan.sl_r.data_ptr(),
                       plan.sr_r.data_ptr(), plan.lsp_r.data_ptr(), plan.dep0.data_ptr(), plan.ready0.data_ptr(),
                       int(plan.ready0.numel()), plan.par_ptr.data_ptr(), plan.par_idx.data_ptr(), queue.data_ptr(),
                       remaining.data_ptr(), counters.data_ptr(), engine.FLOW_MAX_POLLS, Pi.data_ptr(),
                       Pibar.data_ptr(), dts.data_ptr(), dPi.data_ptr(), dPibar.data_ptr(), C * S, D,
                       k["mc"].data_ptr(), k["dl"].data_ptr(), k["ebar"].data_ptr(), k["e"].data_ptr(),
                       k["sl1"].data_ptr(), k["sl2"].data_ptr(), k["leaf"].data_ptr(), pDp.data_ptr(), pSp.data_ptr(),
                       prs, 0, dmc.data_ptr(), dDL.data_ptr(), dEbar.data_ptr(), dE.data_ptr(), dSL1.data_ptr(),
                       dSL2.data_ptr(), dpS.data_ptr(), dpD.data_ptr(), dpS.data_ptr(), S, item_idx.data_ptr(),
                       leaf_state.data_ptr(), tt.tour.data_ptr(), tt.tour_pair.data_ptr(), n_it, S, st)
        if int(counters[2].item()) != 0:
            raise RuntimeError("kb_flow_tangent: a dataflow wait gave up (dependency counts inconsistent)")
        L_range = ()
    else:
        L_range = range(plan.n_levels)
    for L in L_range:
        a, b = plan.level_ptr[L], plan.level_ptr[L + 1]
        if b == a:
            continue
        engine._launch(static, "kb_level_tangent", L, rows_ptr + 4 * a, sp_ptr + 8 * a, b - a, plan.sl.data_ptr(),
                       plan.sr.data_ptr(), plan.lsp.data_ptr(), Pi.data_ptr(), Pibar.data_ptr(), dts.data_ptr(),
                       dPi.data_ptr(), dPibar.data_ptr(), C * S, D, k["mc"].data_ptr(), k["dl"].data_ptr(),
                       k["ebar"].data_ptr(), k["e"].data_ptr(), k["sl1"].data_ptr(), k["sl2"].data_ptr(),
                       k["leaf"].data_ptr(), pDp.data_ptr(), pSp.data_ptr(), prs, 0, dmc.data_ptr(), dDL.data_ptr(),
                       dEbar.data_ptr(), dE.data_ptr(), dSL1.data_ptr(), dSL2.data_ptr(), dpS.data_ptr(),
                       dpD.data_ptr(), dpS.data_ptr(), S, item_idx.data_ptr(), leaf_state.data_ptr(),
                       tt.tour.data_ptr(), _lib.ptr(tt.tour_pair if getattr(static, "_tangent_pairs", True) else None),
                       n_it, S, st)
    roots = dPi.index_select(1, wl["root_row_ids"])
    if return_full:
        return roots, {"dPi": dPi, "dPibar": dPibar, "dE": dE, "dE_s1": dE_s1, "dE_s2": dE_s2, "dEbar": dEbar,
                       "dlog_pS": dpS, "dlog_pD": dpD, "dlog_pL": dpL, "dmax_coupling": dmc, "e_iters": iters}
    return roots
