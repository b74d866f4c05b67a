"""Reference-structured orchestration: the forward and backward passes driven one wrapper call at a
time, exactly as the reference's frozen glue drives its kernels.

This restates, in this library's own code, the call sequence of the reference's
``kbench/core/inference/solver.py:16-142`` (E fixed point, wave loop, NLL),
``kbench/core/inference/forward.py:8-117`` (the per-iteration wave loop with its buffer
ping-pong and aliasing) and ``kbench/api/_implicit_grad.py:28-475`` (reverse wave loop, E-adjoint
BiCGSTAB, theta VJP).  It exercises the drop-in wrappers of ``kbench_b200.kernels`` under the same
contract the reference glue relies on; the fused fast path lives in ``engine.py``.
"""

from __future__ import annotations

import math

import torch

from .kernels.dts_fused import compute_dts_forward
from .kernels.e_step import e_fixed_point_triton, e_step_triton_autograd
from .kernels.wave_backward import (active_mask_from_rhs_absmax_fused, dts_cross_backward_accum_fused,
                                    uniform_cross_pibar_vjp_tree_from_ud_fused, wave_backward_uniform_fused)
from .kernels.wave_step import compute_leaf_initial_wave_step, compute_wave_step
from .params import (as_item_param, as_item_state, extract_parameters_uniform,
                     extract_parameters_weighted_cols)

NEG_INF = float("-inf")


# ----------------------------------------------------------------------------------------------
# forward
# ----------------------------------------------------------------------------------------------

def col_weights_are_uniform(col_weights) -> bool:
    flat = col_weights.detach().reshape(-1)
    return bool(torch.all(flat == flat[0]).item())


def col_weights_uniform_for(static, col_weights) -> bool:
    """col_weights_are_uniform, remembered on ``static`` for the same tensor object at the same
    version (the check reads the device back -- a host synchronisation -- so a solver loop that
    passes one col_weights tensor pays it once, not per call)."""
    c = getattr(static, "_uniform_cols", None)
    if c is not None and c[0] is col_weights and c[1] == col_weights._version:
        return c[2]
    r = col_weights_are_uniform(col_weights)
    static._uniform_cols = (col_weights, col_weights._version, r)
    return r


def logsumexp2(x, dim, keepdim=False):
    m = x.max(dim=dim, keepdim=True).values
    ms = torch.where(m == NEG_INF, torch.zeros_like(m), m)
    tot = torch.exp2(x - ms).sum(dim=dim, keepdim=True)
    pos = tot > 0
    res = torch.where(pos, torch.log2(torch.where(pos, tot, torch.ones_like(tot))), torch.full_like(tot, NEG_INF)) + m
    return res if keepdim else res.squeeze(dim)


def nll_from_root_rows(root_rows, E):
    norm = (1 - torch.exp2(E).mean(dim=-1)).clamp_min(torch.finfo(E.dtype).tiny)
    return (-(logsumexp2(root_rows, dim=-1) - math.log2(root_rows.shape[-1]) - torch.log2(norm))).sum()


def solve_parameters(static, theta, col_weights):
    """(log_pS, log_pD, log_pL, max_coupling, col_log_probs, use_col_weights) as the reference's
    ``solve_e_pi`` derives them (``solver.py:25-44``)."""
    use_col_weights = not col_weights_uniform_for(static, col_weights)
    S = int(static.state_helpers["S"])
    if use_col_weights:
        pS, pD, pL, mc, clp = extract_parameters_weighted_cols(theta.detach(), col_weights.detach(),
                                                               static.state_helpers, statewise=static.statewise,
                                                               itemwise=static.itemwise)
    else:
        pS, pD, pL, mc = extract_parameters_uniform(
            theta.detach(), static.state_helpers["unnorm_row_max"].to(device=theta.device, dtype=theta.dtype),
            statewise=static.statewise, itemwise=static.itemwise)
        clp = theta.new_full((S,), -math.log2(S))
    return pS, pD, pL, mc, clp, use_col_weights


def solve_e(static, pS, pD, pL, mc, clp, use_col_weights, theta, warm_start_E=None):
    so = static.solver_options
    S = int(static.state_helpers["S"])
    shape = (int(static.wave_layout["root_row_ids"].numel()) if static.itemwise else 1, S)
    E0 = warm_start_E.detach().to(theta).contiguous() if warm_start_E is not None else \
        theta.new_full(shape, float(so.e_init))
    sh = static.state_helpers
    return e_fixed_point_triton(E0, log_pS=pS, log_pD=pD, log_pL=pL, max_coupling=mc, col_log_probs=clp,
                                use_col_weights=use_col_weights, node_parent=sh["node_parent"],
                                node_child1=sh["node_child1"], node_child2=sh["node_child2"],
                                max_ancestor_depth=int(sh["max_ancestor_depth"]), max_iter=so.e_max_iter,
                                tol=so.e_tol)


def wave_constants(E, Ebar, E_s1, E_s2, pS, pD, mc, S):
    """The per-item constants the wave kernels take (reference ``forward.py:36-58``)."""
    g = int(E.shape[0])
    e_item = as_item_state(E, S, g)
    return {
        "e": e_item,
        "ebar": as_item_state(Ebar, S, g),
        "mc": as_item_state(mc.squeeze(-1), S, g),
        "dl": 1.0 + as_item_state(pD, S, g) + e_item,
        "sl1": as_item_state(pS, S, g) + as_item_state(E_s2, S, g),
        "sl2": as_item_state(pS, S, g) + as_item_state(E_s1, S, g),
        "leaf": as_item_state(pS, S, g),
        "pD_param": as_item_param(pD, g, S),
        "pS_param": as_item_param(pS, g, S),
    }


def _dts(meta, pi, pibar, sh, k, item_idx, active=None):
    return compute_dts_forward(pi, pibar, meta["sl"], meta["sr"], sh["node_child1"], sh["node_child2"], int(meta["W"]),
                               meta["reduce_idx"], k["pD_param"], k["pS_param"], item_idx=item_idx,
                               log_split_probs=meta.get("log_split_probs"), n_eq1=meta.get("n_eq1"),
                               eq1_reduce_idx=meta.get("eq1_reduce_idx"), ge2_ptr=meta.get("ge2_ptr"),
                               ge2_parent_ids=meta.get("ge2_parent_ids"), ge2_max_fanout=meta.get("ge2_max_fanout"),
                               active_parent_rows=active, item_offset=int(meta["start"]))


def pi_wave_forward(wave_layout, state_helpers, k, col_log_probs, use_col_weights, *, item_idx, pi_iters,
                    pi_residual_out=None):
    """The reference's wave loop (``forward.py:8-117``): per wave, the split reduction then
    ``pi_iters`` Jacobi sweeps ping-ponging between the ``pi`` and ``pibar`` buffers."""
    pi_iters = int(pi_iters)
    if pi_iters < 2 or pi_iters % 2 != 0:
        raise ValueError("pi_iters must be an even integer at least 2")
    C = int(wave_layout["leaf_state_index"].numel())
    sh = state_helpers
    S = int(sh["S"])
    dev = k["e"].device
    pi = torch.empty((C, S), dtype=torch.float32, device=dev)
    pibar = torch.empty((C, S), dtype=torch.float32, device=dev)
    row_max = torch.empty((C,), dtype=torch.float32, device=dev)
    for meta in wave_layout["wave_metas"]:
        ws, W = int(meta["start"]), int(meta["W"])
        has_leaf = "sl" not in meta
        dts_r = None if has_leaf else _dts(meta, pi, pibar, sh, k, item_idx)
        for it in range(pi_iters):
            pi_in, pi_out = (pi, pibar) if it % 2 == 0 else (pibar, pi)
            if it == 0 and not has_leaf:
                continue
            if it == 0:
                compute_leaf_initial_wave_step(pi_out, ws, W, S, k["mc"], k["dl"], k["ebar"], k["e"], k["sl1"],
                                               k["sl2"], col_log_probs, sh["node_child1"], sh["node_child2"],
                                               sh["node_subtree_start"], sh["node_subtree_end"],
                                               wave_layout["leaf_state_index"], k["leaf"], item_idx=item_idx,
                                               use_col_weights=use_col_weights)
                continue
            first_split_step = it == 1 and not has_leaf
            compute_wave_step(dts_r if first_split_step else pi_in, pi_out, pibar, ws, W, S, k["mc"], k["dl"],
                              k["ebar"], k["e"], k["sl1"], k["sl2"], col_log_probs, sh["node_child1"],
                              sh["node_child2"], sh["node_parent"], int(sh["max_ancestor_depth"]), dts_r,
                              leaf_state_idx=wave_layout["leaf_state_index"], leaf_logp=k["leaf"],
                              item_idx=item_idx, pibar_row_max=row_max, store_final_pibar=it == pi_iters - 1,
                              has_leaf_term=has_leaf, input_ws=0 if first_split_step else None,
                              use_col_weights=use_col_weights,
                              pi_residual_out=pi_residual_out if it == pi_iters - 1 else None)
    return pi[wave_layout["root_row_ids"]], pi, pibar, row_max


def solve_e_pi(static, theta, col_weights, *, warm_start_E=None, pi_iters=None, pi_residual_out=None):
    """Reference ``solver.py:16-96``: returns the 13 forward intermediates."""
    static.solver_options.validate()
    pS, pD, pL, mc, clp, ucw = solve_parameters(static, theta, col_weights)
    E, E_s1, E_s2, Ebar = solve_e(static, pS, pD, pL, mc, clp, ucw, theta, warm_start_E)
    S = int(static.state_helpers["S"])
    k = wave_constants(E, Ebar, E_s1, E_s2, pS, pD, mc, S)
    roots, pi, pibar, row_max = pi_wave_forward(
        static.wave_layout, static.state_helpers, k, clp, ucw, item_idx=static.rate_item_idx,
        pi_iters=static.solver_options.pi_iters if pi_iters is None else int(pi_iters),
        pi_residual_out=pi_residual_out)
    return E, E_s1, E_s2, Ebar, roots, pi, pibar, row_max, pS, pD, pL, mc, clp


# ----------------------------------------------------------------------------------------------
# backward
# ----------------------------------------------------------------------------------------------

def _safe_exp2_ratio(a, b):
    neg = a == NEG_INF
    return torch.where(neg, torch.zeros_like(a),
                       torch.exp2(torch.where(neg, torch.zeros_like(a), a) - torch.where(neg, torch.zeros_like(b), b)))


@torch.no_grad()
def bicgstab(Av, b, *, max_iter=500, tol=1e-7, breakdown_tol=1e-30):
    """BiCGSTAB with the reference's stopping and breakdown rules (``_implicit_grad.py:28-94``)."""
    max_iter, tol, breakdown_tol = int(max_iter), float(tol), float(breakdown_tol)
    if max_iter < 1:
        raise ValueError("max_iter must be at least 1")
    if tol <= 0.0:
        raise ValueError("tol must be positive")
    if breakdown_tol <= 0.0:
        raise ValueError("breakdown_tol must be positive")
    x = torch.zeros_like(b)
    r = b - Av(x)
    bnorm = max(float(torch.linalg.vector_norm(b)), 1.0)
    rel = float(torch.linalg.vector_norm(r)) / bnorm
    if rel <= tol:
        return x
    r_hat = r.clone()
    one = torch.ones((), dtype=b.dtype, device=b.device)
    rho_old, alpha, omega = one, one.clone(), one.clone()
    v = torch.zeros_like(b)
    p = torch.zeros_like(b)
    k = 0
    for k in range(1, max_iter + 1):
        rho = torch.dot(r_hat, r)
        if float(rho.abs()) <= breakdown_tol:
            break
        beta = (rho / rho_old) * (alpha / omega)
        p = r + beta * (p - omega * v)
        v = Av(p)
        den = torch.dot(r_hat, v)
        if float(den.abs()) <= breakdown_tol:
            break
        alpha = rho / den
        s = r - alpha * v
        if float(torch.linalg.vector_norm(s)) / bnorm <= tol:
            return x + alpha * p
        t = Av(s)
        tt = torch.dot(t, t)
        if float(tt.abs()) <= breakdown_tol:
            break
        omega = torch.dot(t, s) / tt
        x = x + alpha * p + omega * s
        r = s - omega * t
        rel = float(torch.linalg.vector_norm(r)) / bnorm
        if rel <= tol:
            return x
        if float(omega.abs()) <= breakdown_tol:
            break
        rho_old = rho
    raise RuntimeError(f"E-adjoint BiCGSTAB solve failed after {k} iterations (relative residual {rel:.3e})")


class GradAccumulators:
    """The backward's parameter-cotangent accumulators (reference ``_implicit_grad.py:144-158``)."""

    def __init__(self, E, S, dev):
        g = int(E.shape[0])
        z = lambda: torch.zeros((g, S), device=dev, dtype=torch.float32)  # noqa: E731
        self.pD, self.pS, self.mt = z(), z(), z()
        self.E, self.Ebar, self.E_s1, self.E_s2 = z(), z(), z(), z()
        self.col = torch.zeros((S,), device=dev, dtype=torch.float32)


def root_rhs(Pi, root_ids):
    """Cotangent of the loss w.r.t. the root rows (reference ``_implicit_grad.py:151-158``)."""
    root_Pi = Pi.index_select(0, root_ids)
    return -_safe_exp2_ratio(root_Pi, logsumexp2(root_Pi, dim=-1, keepdim=True))


@torch.no_grad()
def implicit_grad(static, theta, col_weights, saved, *, v_out=None, exact_accumulation=False, cache=None,
                  collect_backward_relres=False):
    """Reference ``_implicit_grad.py:98-370`` followed by :func:`e_adjoint_and_theta_vjp`.

    ``exact_accumulation=False`` reproduces the reference's accumulation exactly: every wave's
    parameter cotangents are added into fp32 running sums (the split kernels add per element
    with atomics).  At large problems those running sums reach ~1e3 while most single-split
    contributions are many orders of magnitude smaller, so fp32 swamping loses ~1e-3 of the
    split sums.  ``exact_accumulation=True`` runs the same kernels but starts each wave's fp32
    partial sums from zero and adds them into fp64 totals (the accuracy the fused engine gets
    from its fp64 accumulators).

    ``cache`` (a dict) receives the point cache of the exact-Hessian HVP (``newton/ggn.py:152-162``,
    ``newton/hvp_exact.py:37-45``): ``waves`` -- per wave in the order processed (reverse wave
    order) ``ws, W, v`` (adjoint rows, zero on inactive rows), ``dts_r, active_mask, has_splits,
    has_leaf_term, meta`` --, ``accum`` (the column cotangent accumulators) and ``wE`` (the
    E-side adjoint).

    ``collect_backward_relres`` (reference ``_implicit_grad.py:117,189-195,263-288,355``): the
    reverse wave loop runs as usual, then ``(relres, vk_mag)`` is returned instead of the
    gradients -- per family the largest ``|last Neumann term| / |v|`` and the largest ``|v|`` over
    its active rows."""
    so = static.solver_options
    wl, sh = static.wave_layout, static.state_helpers
    Pi, Pibar = saved["pi_wave"], saved["pibar_wave"]
    C, S = int(Pi.shape[0]), int(Pi.shape[1])
    dev = Pi.device
    E = saved["E"]
    ucw = not col_weights_are_uniform(col_weights)
    k = wave_constants(E, saved["Ebar"], saved["E_s1"], saved["E_s2"], saved["log_pS"], saved["log_pD"],
                       saved["max_coupling"], S)
    acc = torch.zeros((C, S), device=dev, dtype=torch.float32)
    g = GradAccumulators(E, S, dev)
    if exact_accumulation:
        g_total = {n: torch.zeros((S,), device=dev, dtype=torch.float64)
                   for n in ("pD", "pS", "mt", "E", "Ebar", "E_s1", "E_s2", "col")}
    roots = wl["root_row_ids"]
    acc.index_copy_(0, roots, root_rhs(Pi, roots))
    item_idx = static.rate_item_idx
    leaf_state = wl["leaf_state_index"].to(device=dev, dtype=torch.int32).contiguous()
    chunk = 64 if exact_accumulation else None
    if collect_backward_relres:
        row_item = wl["item_idx"].to(device=dev, dtype=torch.long)
        n_fam = int(row_item.max().item()) + 1 if row_item.numel() else 0
        relres = torch.zeros(n_fam, device=dev, dtype=torch.float32)
        vk_mag = torch.zeros(n_fam, device=dev, dtype=torch.float32)

    def flush():
        for n in ("pD", "pS", "mt", "E", "Ebar", "E_s1", "E_s2"):
            g_total[n] += getattr(g, n)[0].double()
            getattr(g, n).zero_()
        g_total["col"] += g.col.double()
        g.col.zero_()

    for meta in reversed(wl["wave_metas"]):
        ws, W = int(meta["start"]), int(meta["W"])
        rhs_k = acc[ws:ws + W]
        active = active_mask_from_rhs_absmax_fused(rhs_k, so.adjoint_pruning_threshold,
                                                   use_pruning=bool(so.use_adjoint_pruning)).contiguous()
        has_splits = "sl" in meta
        dts_r = _dts(meta, Pi, Pibar, sh, k, item_idx, active) if has_splits else None
        v_k = torch.empty((W, S), device=dev, dtype=torch.float32)
        row_blocks = [(0, W)] if chunk is None else [(a, min(a + chunk, W)) for a in range(0, W, chunk)]
        for a, b in row_blocks:
            out = wave_backward_uniform_fused(
                Pi, Pibar, ws + a, b - a, S, None if dts_r is None else dts_r[a:b], rhs_k[a:b], k["mc"], k["dl"],
                k["ebar"], k["e"], k["sl1"], k["sl2"], saved["col_log_probs"], sh["node_child1"], sh["node_child2"],
                None, neumann_terms=so.neumann_terms, leaf_state_idx=leaf_state, leaf_logp=k["leaf"],
                has_leaf_term=not has_splits, active_mask=active[a:b], node_parent=sh["node_parent"],
                max_ancestor_depth=int(sh["max_ancestor_depth"]), pibar_row_max=saved["pibar_row_max"],
                item_idx=item_idx, item_indexed_consts=True, compact_level_ptr=sh["compact_level_ptr"],
                compact_level_parents=sh["compact_level_parents"], compact_level_child1=sh["compact_level_child1"],
                compact_level_child2=sh["compact_level_child2"], grad_col_log_probs=g.col, use_col_weights=ucw,
                self_loop_solver=so.self_loop_solver, return_last_increment=collect_backward_relres)
            vb, aw0, aw1, aw2, aw345, aw3, aw4 = out[:7]
            if collect_backward_relres:
                wave_item = row_item[ws + a:ws + b]
                on = active[a:b].reshape(b - a, -1).ne(0).any(dim=1)
                vk_norm = torch.where(on, vb.float().norm(dim=1), torch.zeros_like(vb[:, 0]))
                vk_mag.scatter_reduce_(0, wave_item, vk_norm, reduce="amax", include_self=True)
                if out[7] is not None:
                    relres.scatter_reduce_(0, wave_item, out[7].float(), reduce="amax", include_self=True)
            v_k[a:b] = vb
            dbg = getattr(static, "_debug_sums", None)
            if dbg is not None:
                for name, t in (("aw0", aw0), ("aw1", aw1), ("aw2", aw2), ("aw3", aw3), ("aw4", aw4), ("aw345", aw345)):
                    dbg[name] = dbg.get(name, 0) + t.double().sum(dim=0)
            g.pD[0] += aw0.sum(dim=0)
            g.pS[0] += aw345.sum(dim=0)
            g.E[0] += (aw0 + aw2).sum(dim=0)
            g.Ebar[0] += aw1.sum(dim=0)
            g.E_s1[0] += aw4.sum(dim=0)
            g.E_s2[0] += aw3.sum(dim=0)
            g.mt[0] += aw2.sum(dim=0)
            if exact_accumulation:
                flush()
        if v_out is not None:
            v_out[ws:ws + W][active] = v_k[active]
        if cache is not None:
            row_on = active.reshape(W, -1).any(dim=1)
            cache.setdefault("waves", []).append(dict(
                ws=ws, W=W, v=torch.where(row_on[:, None], v_k, torch.zeros_like(v_k)), dts_r=dts_r,
                active_mask=active, has_splits=has_splits, has_leaf_term=not has_splits, meta=meta))
        if has_splits:
            n_split = int(meta["sl"].numel())
            split_blocks = [(0, n_split)] if chunk is None else [(a, min(a + chunk, n_split))
                                                                   for a in range(0, n_split, chunk)]
            for a, b in split_blocks:
                sl_c, sr_c, red_c = meta["sl"][a:b], meta["sr"][a:b], meta["reduce_idx"][a:b]
                ud, A, side, _, _ = dts_cross_backward_accum_fused(
                    Pi, Pibar, v_k, ws, sl_c, sr_c, red_c, meta["log_split_probs"][a:b], k["pD_param"],
                    k["pS_param"], sh["node_child1"], sh["node_child2"], acc, S, active_mask=active,
                    merge_s_term=True, grad_log_pD=g.pD, grad_log_pS=g.pS, grad_mt=g.mt,
                    accum_param_reductions=True, accum_mt_reduction=True, output_pibar_ud=True,
                    output_pibar_side_active=True, pibar_side_threshold=so.pibar_side_threshold,
                    mt_squeezed=k["mc"], pibar_row_max=saved["pibar_row_max"],
                    skip_inactive_pibar_output_zero=True, item_idx=item_idx)
                uniform_cross_pibar_vjp_tree_from_ud_fused(
                    Pi, saved["col_log_probs"], ud, A, sl_c, sr_c, acc, S, active_mask=active, reduce_idx=red_c,
                    pibar_row_max=saved["pibar_row_max"], skip_zero_sides=True, side_active=side,
                    compact_level_ptr=sh["compact_level_ptr"], compact_level_parents=sh["compact_level_parents"],
                    compact_level_child1=sh["compact_level_child1"],
                    compact_level_child2=sh["compact_level_child2"], grad_col_log_probs=g.col, use_col_weights=ucw,
                    side_active_threshold=so.pibar_side_threshold)
                if exact_accumulation:
                    flush()
    if collect_backward_relres:
        return relres, vk_mag
    if exact_accumulation:
        for n in ("pD", "pS", "mt", "E", "Ebar", "E_s1", "E_s2"):
            getattr(g, n)[0] = g_total[n].float()
        g.col.copy_(g_total["col"].float())
    static._last_acc = acc
    out = e_adjoint_and_theta_vjp(static, theta, col_weights, saved, g, int(roots.numel()), ucw)
    if cache is not None:
        cache["accum"] = g
        cache["wE"] = static._last_e_adjoint
    return out


DEVICE_E_ADJOINT = True  # one shared E row: the whole solve in one launch (kb_e_adjoint_solve)


def _e_adjoint_one_launch(static, theta, col_weights, saved, g, n_fam, use_col_weights, topo, check=True):
    """:func:`e_adjoint_and_theta_vjp` for one shared E row: the right-hand side, the BiCGSTAB
    solve and the E step's parameter VJP run in ONE kernel (``kb_e_adjoint_solve``); what is left
    here is the VJP of the parameter extraction, with the same terms as the general path.  With
    ``check=False`` the solve's convergence status is kept on ``static._pending_e_adjoint`` for
    :func:`check_pending_e_adjoint` instead of being read back now."""
    from .kernels.e_step import _as_item_state_ad, e_adjoint_check, e_adjoint_solve
    so = static.solver_options
    sh = static.state_helpers
    S = int(sh["S"])
    wE, gp, status, rel = e_adjoint_solve(saved["E"], saved["log_pS"], saved["log_pD"], saved["log_pL"],
                                          saved["max_coupling"], saved["col_log_probs"], *topo, g.E, g.Ebar,
                                          g.E_s1, g.E_s2, n_fam=n_fam, max_iter=so.bicgstab_max_iter,
                                          tol=so.bicgstab_tol, breakdown_tol=so.bicgstab_breakdown_tol,
                                          use_col_weights=use_col_weights, check=False)
    if check:
        e_adjoint_check(status, rel)
    else:
        pending = getattr(static, "_pending_e_adjoint", None)
        if pending is None:
            pending = static._pending_e_adjoint = []
        pending.append((status, rel))
    static._last_e_adjoint = wE
    theta_req = theta.detach().requires_grad_(True)
    col_req = col_weights.detach().requires_grad_(True)
    with torch.enable_grad():
        pS, pD, pL, mt, clp = extract_parameters_weighted_cols(theta_req, col_req, sh, statewise=static.statewise,
                                                               itemwise=static.itemwise,
                                                               uniform_fast=not use_col_weights)
        loss = ((as_item_param(pS, 1, S) * g.pS).sum() + (as_item_param(pD, 1, S) * g.pD).sum()
                + (mt * g.mt.reshape(mt.shape)).sum() + (clp * g.col).sum()
                + (_as_item_state_ad(pS, S, 1) * gp[0:1]).sum() + (_as_item_state_ad(pD, S, 1) * gp[1:2]).sum()
                + (_as_item_state_ad(pL, S, 1) * gp[2:3]).sum() + (_as_item_state_ad(mt, S, 1) * gp[3:4]).sum()
                + (clp.contiguous().reshape(-1) * gp[4]).sum())
        grad_theta, grad_col = torch.autograd.grad(loss, (theta_req, col_req))
    return grad_theta, grad_col


def check_pending_e_adjoint(static) -> None:
    """Read the convergence status of the E-adjoint solves run with ``check=False`` on ``static``
    (one host synchronisation) and raise the reference's ``RuntimeError`` for one that failed."""
    from .kernels.e_step import e_adjoint_check
    pending = getattr(static, "_pending_e_adjoint", None)
    if not pending:
        return
    static._pending_e_adjoint = []
    for status, rel in pending:
        e_adjoint_check(status, rel)


def e_adjoint_and_theta_vjp(static, theta, col_weights, saved, g, n_fam, use_col_weights, check=True):
    """The accumulated cotangents are kept on ``static._last_grad_acc`` for inspection.
    ``check=False`` defers the one-launch solve's convergence check (:func:`check_pending_e_adjoint`).

    Reference ``_implicit_grad.py:373-475``: solve ``(I - J_E^T) w = q`` with BiCGSTAB, one E-step
    VJP kernel per matvec, then the theta / column-weight VJP through the parameter extraction."""
    so = static.solver_options
    sh = static.state_helpers
    static._last_grad_acc = g
    topo = (sh["node_parent"], sh["node_child1"], sh["node_child2"], int(sh["max_ancestor_depth"]))
    E_star = saved["E"]
    if DEVICE_E_ADJOINT and E_star.shape[0] == 1 and E_star.is_cuda:
        return _e_adjoint_one_launch(static, theta, col_weights, saved, g, n_fam, use_col_weights, topo, check)
    E_req = E_star.detach().requires_grad_(True)
    with torch.enable_grad():
        E_from_E, Es1_from_E, Es2_from_E, Ebar_from_E = e_step_triton_autograd(
            E_req, saved["log_pS"], saved["log_pD"], saved["log_pL"], saved["max_coupling"], saved["col_log_probs"],
            *topo, use_col_weights=use_col_weights)
        norm = (1 - torch.exp2(E_req).mean(dim=-1)).clamp_min(torch.finfo(E_req.dtype).tiny)
        denom = torch.log2(norm)
        direct = denom.sum() if E_req.shape[0] == n_fam else (n_fam * denom).sum()
        (aux,) = torch.autograd.grad((direct, Es1_from_E, Es2_from_E, Ebar_from_E), E_req,
                                     grad_outputs=(torch.ones_like(direct), g.E_s1, g.E_s2, g.Ebar),
                                     retain_graph=True)
    q = (g.E + aux).reshape(-1)
    shape = E_star.shape

    def AG(w):
        wE = w.view(shape).contiguous()
        with torch.enable_grad():
            (gE,) = torch.autograd.grad(E_from_E, E_req, grad_outputs=wE.clone(), retain_graph=True)
        return (wE - gE).reshape(-1)

    wE = bicgstab(AG, q, max_iter=so.bicgstab_max_iter, tol=so.bicgstab_tol,
                  breakdown_tol=so.bicgstab_breakdown_tol).view(shape)
    static._last_e_adjoint = wE
    theta_req = theta.detach().requires_grad_(True)
    col_req = col_weights.detach().requires_grad_(True)
    with torch.enable_grad():
        pS, pD, pL, mt, clp = extract_parameters_weighted_cols(theta_req, col_req, sh, statewise=static.statewise,
                                                               itemwise=static.itemwise,
                                                               uniform_fast=not use_col_weights)
        S = int(sh["S"])
        rows = int(E_star.shape[0])
        loss = ((as_item_param(pS, rows, S) * g.pS).sum() + (as_item_param(pD, rows, S) * g.pD).sum()
                + (mt * g.mt.reshape(mt.shape)).sum() + (clp * g.col).sum())
        E_p, _, _, Ebar_p = e_step_triton_autograd(E_star.detach(), pS, pD, pL, mt, clp, *topo,
                                                   use_col_weights=use_col_weights)
        grad_theta, grad_col = torch.autograd.grad((loss, Ebar_p, E_p), (theta_req, col_req),
                                                   grad_outputs=(torch.ones_like(loss), g.Ebar, wE))
    return grad_theta, grad_col
