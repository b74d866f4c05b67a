"""CPU oracle for the analytic exact-Hessian HVP -- TEST INFRASTRUCTURE ONLY.

A numpy float32 restatement of the reference's forward-over-reverse Hessian-vector product:
``newton/hvp_exact.py:37-375`` (``build_point_cache`` / ``make_exact_hvp``) with its second-order
contraction kernels ``kbench/core/kernels/wave_so.py:37-250`` (``_wave_so_kernel``),
``kbench/core/kernels/dts_so.py:24-230`` (``_dts_split_so_kernel``, ``_dts_tree_so_kernel``) and
``kbench/core/kernels/e_step_so.py:23-185`` (``_e_step_so_prepare/finalize_kernel``), over the
first-order pieces of ``kb_oracle`` (the reverse wave loop, the E-step VJP, BiCGSTAB) and the
tangent of ``kb_oracle_tangent``.  Only ``tests/`` may import it; the CUDA path never calls into
this file.  Pinned by ``tests/golden/make_golden.py --hvp`` (the reference's own HVP run under
``TRITON_INTERPRET=1`` on the CPU).
"""

from __future__ import annotations

import numpy as np

from .kb_oracle import (F32, LN2, NEG_INF, Tree, _f, _safe, backward_accumulators, bicgstab, dts_cross_backward,
                        e_adjoint_and_theta_vjp, e_step_forward, e_step_vjp, extract_parameters_vjp, lse_rows,
                        pibar_vjp_tree, wave_backward)
from .kb_oracle_tangent import dts_tangent, jvp_root_scores

_L = F32(LN2)


def _exp2(x):
    with np.errstate(over="ignore"):
        return np.exp2(x).astype(F32)


def wave_backward_so(Pi, dPi, Pibar, dPibar, v, ws, W, row_max_all, consts, dc, tree: Tree, *, dts_r=None,
                     d_dts=None, leaf_state=None, leaf_logp=None, dleaf_logp=None, d_rhs=None):
    """``wave_so.py:37-250``: tangent of the self-loop J^T application and of the parameter buckets
    at FIXED adjoint ``v`` [W,S] (every row of the wave, inactive ones carry v = 0).  Returns
    (d_Av [W,S] -- with the wave's rows of ``d_rhs`` folded in when given --, d_aw0, d_aw1, d_aw2,
    d_aw345, d_aw3, d_aw4)."""
    S = tree.S
    rows = ws + np.arange(W)
    pi, dpi = Pi[rows], dPi[rows]
    pib, dpib = Pibar[rows], dPibar[rows]
    v = _f(v)
    rm = row_max_all[rows]
    rms = _safe(rm)[:, None]
    p_prime = np.where(pi != NEG_INF, _exp2(pi - rms), F32(0.0)).astype(F32)
    dp_prime = (_L * p_prime * dpi).astype(F32)
    row_sum = p_prime.sum(axis=-1, dtype=F32)[:, None]
    drow_sum = dp_prime.sum(axis=-1, dtype=F32)[:, None]
    anc = tree.ancestor_sum(p_prime)
    danc = tree.ancestor_sum(dp_prime)
    denom = (row_sum - anc).astype(F32)
    with np.errstate(divide="ignore"):
        inv_denom = np.where(denom > 0, F32(1.0) / np.where(denom > 0, denom, 1), F32(0.0)).astype(F32)
    ddenom = (drow_sum - danc).astype(F32)

    def g(rows_, which):
        return tree.gather_child(rows_, which)

    def dg(rows_, which):
        ok, idx = (tree.c1_valid, tree.c1_safe) if which == 1 else (tree.c2_valid, tree.c2_safe)
        return np.where(ok, rows_[..., idx], F32(0.0)).astype(F32)

    t = [(consts["dl"] + pi).astype(F32), (pi + consts["ebar"]).astype(F32), (pib + consts["e"]).astype(F32),
         (consts["sl1"] + g(pi, 1)).astype(F32), (consts["sl2"] + g(pi, 2)).astype(F32)]
    dt = [(dc["dDL"] + dpi).astype(F32), (dpi + dc["dEbar"]).astype(F32), (dpib + dc["dE"]).astype(F32),
          (dc["dSL1"] + dg(dpi, 1)).astype(F32), (dc["dSL2"] + dg(dpi, 2)).astype(F32)]
    t5 = np.full(pi.shape, NEG_INF, dtype=F32)
    dt5 = np.zeros(pi.shape, dtype=F32)
    if leaf_state is not None:
        ok = np.nonzero(leaf_state >= 0)[0]
        t5[ok, leaf_state[ok]] = _f(leaf_logp)[leaf_state[ok]]
        dt5[ok, leaf_state[ok]] = _f(dleaf_logp)[leaf_state[ok]]
    t.append(t5)
    dt.append(dt5)
    m = t[0]
    for x in t[1:]:
        m = np.maximum(m, x)
    ms = _safe(m)
    e = [_exp2(x - ms) for x in t]
    lsum = (e[0] + e[1] + e[2] + e[3] + e[4] + e[5]).astype(F32)
    with np.errstate(divide="ignore"):
        inv_sum = np.where(lsum > 0, F32(1.0) / np.where(lsum > 0, lsum, 1), F32(0.0)).astype(F32)
    w = [(x * inv_sum).astype(F32) for x in e]
    dlse = (w[0] * dt[0] + w[1] * dt[1] + w[2] * dt[2] + w[3] * dt[3] + w[4] * dt[4] + w[5] * dt[5]).astype(F32)
    dw = [(_L * w[k] * (dt[k] - dlse)).astype(F32) for k in range(6)]
    if dts_r is not None:
        dts_r = _f(dts_r)
        with np.errstate(divide="ignore", invalid="ignore"):
            dts_l = np.where(lsum > 0, np.log2(np.where(lsum > 0, lsum, 1)) + m, NEG_INF).astype(F32)
            pm = np.maximum(dts_l, dts_r)
            pms = _safe(pm)
            pi_new = (np.log2(_exp2(dts_l - pms) + _exp2(dts_r - pms)) + pm).astype(F32)
            w_L = np.where(dts_l != NEG_INF, _exp2(dts_l - pi_new), F32(0.0)).astype(F32)
        ok = (dts_r != NEG_INF) & (dts_l != NEG_INF)
        dw_L = np.where(ok, _L * w_L * (F32(1.0) - w_L) * (dlse - _f(d_dts)), F32(0.0)).astype(F32)
    else:
        w_L = np.ones(pi.shape, dtype=F32)
        dw_L = np.zeros(pi.shape, dtype=F32)
    da = [(v * (dw_L * w[k] + w_L * dw[k])).astype(F32) for k in range(6)]
    coeff = (w_L * w[2] * inv_denom).astype(F32)
    dcoeff = ((dw_L * w[2] + w_L * dw[2]) * inv_denom - coeff * inv_denom * ddenom).astype(F32)
    u = (v * coeff).astype(F32)
    du = (v * dcoeff).astype(F32)
    A = u.sum(axis=-1, dtype=F32)[:, None]
    dA = du.sum(axis=-1, dtype=F32)[:, None]
    sub = tree.subtree_sums_inplace(u.copy())
    dsub = tree.subtree_sums_inplace(du.copy())
    d_diag = (dw_L * (w[0] + w[1]) + w_L * (dw[0] + dw[1])).astype(F32)
    d_out = (v * d_diag + dp_prime * (A - sub) + p_prime * (dA - dsub)).astype(F32)
    if d_rhs is not None:
        d_out = (d_out + d_rhs[rows]).astype(F32)
    d_sl1 = (v * (dw_L * w[3] + w_L * dw[3])).astype(F32)
    d_sl2 = (v * (dw_L * w[4] + w_L * dw[4])).astype(F32)
    for j in range(W):
        np.add.at(d_out[j], tree.c1[tree.c1_valid], d_sl1[j][tree.c1_valid])
        np.add.at(d_out[j], tree.c2[tree.c2_valid], d_sl2[j][tree.c2_valid])
    return (d_out, da[0], da[1], da[2], (da[3] + da[4] + da[5]).astype(F32), da[3], da[4])


def dts_backward_so(Pi, dPi, Pibar, dPibar, v, ws, meta, pD, pS, dpD, dpS, mt, dmt, row_max_all, tree: Tree,
                    d_rhs, d_grad_pD, d_grad_pS, d_grad_mt, d_grad_col):
    """``dts_so.py:24-230``: tangent of the split cotangents and of the Pibar VJP trees at FIXED
    adjoint ``v`` [W,S]; accumulates into ``d_rhs`` [C,S] and the ``d_grad_*`` vectors."""
    S = tree.S
    sl = np.asarray(meta["sl"], dtype=np.int64)
    sr = np.asarray(meta["sr"], dtype=np.int64)
    red = np.asarray(meta["reduce_idx"], dtype=np.int64)
    lsp = meta.get("log_split_probs")
    N = sl.shape[0]
    lsp = np.zeros(N, F32) if lsp is None else _f(lsp).reshape(-1)
    pD, pS, dpD, dpS, mt, dmt = (_f(x).reshape(-1) for x in (pD, pS, dpD, dpS, mt, dmt))

    def g(row, which):
        return tree.gather_child(row, which)

    def dg(row, which):
        ok, idx = (tree.c1_valid, tree.c1_safe) if which == 1 else (tree.c2_valid, tree.c2_safe)
        return np.where(ok, row[idx], F32(0.0)).astype(F32)

    ud = np.zeros((2 * N, S), dtype=F32)
    dud = np.zeros((2 * N, S), dtype=F32)
    m1, m2 = tree.c1_valid, tree.c2_valid
    for n in range(N):
        l, r, w = sl[n], sr[n], red[n]
        pil, pir, pbl, pbr = Pi[l], Pi[r], Pibar[l], Pibar[r]
        dpl, dpr, dbl, dbr = dPi[l], dPi[r], dPibar[l], dPibar[r]
        pip, dpip = Pi[ws + w], dPi[ws + w]
        vv = _f(v[w])
        d = [(lsp[n] + pD + pil + pir).astype(F32), (lsp[n] + pil + pbr).astype(F32),
             (lsp[n] + pir + pbl).astype(F32), (lsp[n] + pS + g(pil, 1) + g(pir, 2)).astype(F32),
             (lsp[n] + pS + g(pir, 1) + g(pil, 2)).astype(F32)]
        dd = [(dpD + dpl + dpr).astype(F32), (dpl + dbr).astype(F32), (dpr + dbl).astype(F32),
              (dpS + dg(dpl, 1) + dg(dpr, 2)).astype(F32), (dpS + dg(dpr, 1) + dg(dpl, 2)).astype(F32)]
        fin = pip != NEG_INF
        wk = [np.where(fin, _exp2(x - pip), F32(0.0)).astype(F32) for x in d]
        vd1 = (vv * wk[1]).astype(F32)
        vd2 = (vv * wk[2]).astype(F32)
        dvd = [(vv * _L * wk[k] * (dd[k] - dpip)).astype(F32) for k in range(5)]
        d_rhs[l] += (dvd[0] + dvd[1]).astype(F32)
        d_rhs[r] += (dvd[0] + dvd[2]).astype(F32)
        np.add.at(d_rhs[l], tree.c1[m1], dvd[3][m1])
        np.add.at(d_rhs[r], tree.c1[m1], dvd[4][m1])
        np.add.at(d_rhs[r], tree.c2[m2], dvd[3][m2])
        np.add.at(d_rhs[l], tree.c2[m2], dvd[4][m2])
        f_l = np.where(pbl != NEG_INF, _exp2(row_max_all[l] + mt - pbl), F32(0.0)).astype(F32)
        f_r = np.where(pbr != NEG_INF, _exp2(row_max_all[r] + mt - pbr), F32(0.0)).astype(F32)
        ud[n] = vd2 * f_l
        ud[N + n] = vd1 * f_r
        dud[n] = (dvd[2] * f_l + vd2 * _L * f_l * (dmt - dbl)).astype(F32)
        dud[N + n] = (dvd[1] * f_r + vd1 * _L * f_r * (dmt - dbr)).astype(F32)
        d_grad_pD += dvd[0]
        d_grad_pS += (dvd[3] + dvd[4]).astype(F32)
        d_grad_mt += (dvd[1] + dvd[2]).astype(F32)
    for row in range(2 * N):
        n = row if row < N else row - N
        child = sl[n] if row < N else sr[n]
        A = ud[row].sum(dtype=F32)
        dA = dud[row].sum(dtype=F32)
        sub = tree.subtree_sums_inplace(ud[row].copy())
        dsub = tree.subtree_sums_inplace(dud[row].copy())
        rms = _safe(row_max_all[child])
        pc = Pi[child]
        pp = np.where(pc != NEG_INF, _exp2(pc - rms), F32(0.0)).astype(F32)
        dpp = (_L * pp * dPi[child]).astype(F32)
        contrib = (dpp * (A - sub) + pp * (dA - dsub)).astype(F32)
        d_rhs[child] += contrib
        d_grad_col += contrib


def e_step_backward_so(E, E_new, E_s1, E_s2, Ebar, pS, pD, pL, tree: Tree, g_new, g_ebar, dE, dE_new, dE_s1,
                       dE_s2, dEbar, dpS, dpD, dpL):
    """``e_step_so.py:23-185`` (uniform column weights): the tangent of the E-step VJP outputs at
    FIXED cotangents ``(g_new, g_ebar)`` along the primal tangent.  Returns (d_grad_E, d_grad_pS,
    d_grad_pD, d_grad_pL, d_grad_mc, d_grad_col)."""
    E, E_new, E_s1, E_s2, Ebar = (_f(x).reshape(-1) for x in (E, E_new, E_s1, E_s2, Ebar))
    pS, pD, pL, g_new, g_ebar = (_f(x).reshape(-1) for x in (pS, pD, pL, g_new, g_ebar))
    dE, dE_new, dE_s1, dE_s2, dEbar = (_f(x).reshape(-1) for x in (dE, dE_new, dE_s1, dE_s2, dEbar))
    dpS, dpD, dpL = (_f(x).reshape(-1) for x in (dpS, dpD, dpL))
    rm = E.max()
    rms = F32(0.0) if rm == NEG_INF else rm
    t = [(pS + E_s1 + E_s2).astype(F32), (pD + F32(2.0) * E).astype(F32), (E + Ebar).astype(F32), pL]
    dt = [(dpS + dE_s1 + dE_s2).astype(F32), (dpD + F32(2.0) * dE).astype(F32), (dE + dEbar).astype(F32), dpL]
    q = [(g_new * _exp2(x - E_new)).astype(F32) for x in t]
    dq = [(_L * q[k] * (dt[k] - dE_new)).astype(F32) for k in range(4)]
    d_grad_E = (F32(2.0) * dq[1] + dq[2]).astype(F32)
    np.add.at(d_grad_E, tree.c1[tree.c1_valid], dq[0][tree.c1_valid])
    np.add.at(d_grad_E, tree.c2[tree.c2_valid], dq[0][tree.c2_valid])
    r = _exp2(E - rms)
    dr = (_L * r * dE).astype(F32)
    row_sum = r.sum(dtype=F32)
    drow_sum = dr.sum(dtype=F32)
    anc = tree.ancestor_sum(r)
    danc = tree.ancestor_sum(dr)
    denom = (row_sum - anc).astype(F32)
    ddenom = (drow_sum - danc).astype(F32)
    pos = denom > 0
    safe = np.where(pos, denom, F32(1.0))
    wbar = (q[2] + g_ebar).astype(F32)
    u = np.where(pos, wbar / safe, F32(0.0)).astype(F32)
    du = np.where(pos, (dq[2] - u * ddenom) / safe, F32(0.0)).astype(F32)
    tot, dtot = u.sum(dtype=F32), du.sum(dtype=F32)
    excl = tree.subtree_sums_inplace(u.copy())
    dexcl = tree.subtree_sums_inplace(du.copy())
    d_pv = (dr * (tot - excl) + r * (dtot - dexcl)).astype(F32)
    return ((d_grad_E + d_pv).astype(F32), dq[0], dq[1], dq[3], dq[2], d_pv)


def point_cache(static: dict, theta, col_weights, saved: dict) -> dict:
    """``hvp_exact.py:37-45`` ``build_point_cache``: the reverse wave loop with its per-wave adjoint
    state recorded, the accumulators and the E-side adjoint ``wE`` (plus the gradient)."""
    waves: list = []
    acc = backward_accumulators(static, saved, cache=waves)
    n_fam = int(np.asarray(static["wave_layout"]["root_row_ids"]).shape[0])
    out: dict = {}
    gt, gc = e_adjoint_and_theta_vjp(static, theta, col_weights, saved, Tree(static["state_helpers"]), acc["E"],
                                     acc["Ebar"], acc["E_s1"], acc["E_s2"], acc["pD"], acc["pS"], acc["mt"],
                                     acc["col"], n_fam=n_fam, out=out)
    return {"waves": waves, "acc": acc, "wE": out["wE"], "grad_theta": gt, "grad_col": gc}


def head_hvp(theta, u, cot):
    """Second-order term of the smooth parameter head (``hvp_exact.py:167-185, 365-373``): the
    Hessian of ``phi1 = sum_s cot_s . log2softmax([0, theta_s])`` (cotangents on log_pS, log_pD,
    log_pL and max_coupling = log_pT + const) applied to ``u``.  With ``p = softmax2([0, theta_s])``
    the Hessian of ``log2softmax_k`` in the logits is ``-ln2 (diag p - p p^T)``, so
    ``H u = -ln2 (sum_k cot_k) (p * [0,u] - p (p . [0,u]))`` restricted to the theta entries."""
    theta = np.asarray(theta, dtype=np.float64)
    S = theta.shape[0]
    u = np.asarray(u, dtype=np.float64).reshape(S, 3)
    logits = np.concatenate([np.zeros((S, 1)), theta], axis=1)
    p = np.exp2(logits - logits.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    ul = np.concatenate([np.zeros((S, 1)), u], axis=1)
    c = np.stack([np.asarray(x, dtype=np.float64).reshape(-1) for x in cot], axis=1).sum(axis=1, keepdims=True)
    h = -LN2 * c * (p * ul - p * (p * ul).sum(axis=1, keepdims=True))
    return h[:, 1:]


def hvp(static: dict, theta, col_weights, saved: dict, u, *, cache: dict | None = None, self_iters=None,
        debug_out: dict | None = None):
    """``hvp_exact.py:64-375`` ``make_exact_hvp(...)(u)``: one tangent forward sweep, the
    tangent-adjoint sweep over the cached waves (second-order contraction at fixed v, then the
    same Neumann solve seeded with it, then the split cotangents of the new adjoint and the
    split second-order term), the E side (tangent of the E-adjoint right-hand side, a BiCGSTAB solve
    with the same operator, the E step's parameter cotangent tangents) and the smooth head.
    Returns ``H u`` flattened ``[3S]``."""
    sh, wl, so = static["state_helpers"], static["wave_layout"], static["solver_options"]
    tree = Tree(sh)
    S = tree.S
    if cache is None:
        cache = point_cache(static, theta, col_weights, saved)
    acc, wE = cache["acc"], cache["wE"]
    if self_iters is None:
        self_iters = int(so["pi_iters"])
    u = _f(u).reshape(S, 3)
    Pi, Pibar = _f(saved["pi_wave"]), _f(saved["pibar_wave"])
    E, Ebar = _f(saved["E"]).reshape(-1), _f(saved["Ebar"]).reshape(-1)
    E_s1, E_s2 = _f(saved["E_s1"]).reshape(-1), _f(saved["E_s2"]).reshape(-1)
    pS, pD, pL = (_f(saved[k]).reshape(-1) for k in ("log_pS", "log_pD", "log_pL"))
    mc = _f(saved["max_coupling"]).reshape(-1)
    col_logp = _f(saved["col_log_probs"]).reshape(-1)
    row_max = _f(saved["pibar_row_max"])
    C = Pi.shape[0]
    consts = {"dl": (F32(1.0) + pD + E).astype(F32), "ebar": Ebar, "e": E,
              "sl1": (pS + E_s2).astype(F32), "sl2": (pS + E_s1).astype(F32), "mc": mc}
    t_root, dPi, dPibar, dc = jvp_root_scores(static, theta, u, saved, self_iters=self_iters)
    raw = dc["raw"]
    roots = np.asarray(wl["root_row_ids"], dtype=np.int64)
    root_Pi = Pi[roots]
    lse = lse_rows(root_Pi)[:, None]
    q = np.where(root_Pi != NEG_INF, _exp2(np.where(root_Pi != NEG_INF, root_Pi, 0) - lse), F32(0.0)).astype(F32)
    d_seed = (-_L * q * (t_root - (q * t_root).sum(axis=-1, keepdims=True, dtype=F32))).astype(F32)
    d_rhs = np.zeros((C, S), dtype=F32)
    d_rhs[roots] = d_seed
    z = lambda: np.zeros(S, dtype=F32)  # noqa: E731
    d_gpD, d_gpS, d_gE, d_gEbar, d_gEs1, d_gEs2, d_gmc, d_gcol = (z() for _ in range(8))
    leaf_state_all = np.asarray(wl["leaf_state_index"], dtype=np.int64)
    for wave in cache["waves"]:  # already in reverse wave order
        ws, W, meta = wave["ws"], wave["W"], wave["meta"]
        v_k, dts_r, act = wave["v"], wave["dts_r"], wave["active"]
        d_dts = None
        if dts_r is not None:
            d_dts = dts_tangent(Pi, Pibar, dPi, dPibar, meta, pD, pS, dc["dpd_param"], dc["dps_param"], dts_r, tree)
        ls = None if wave["has_splits"] else leaf_state_all[ws:ws + W]
        c_out = wave_backward_so(Pi, dPi, Pibar, dPibar, v_k, ws, W, row_max, consts, dc, tree, dts_r=dts_r,
                                 d_dts=d_dts, leaf_state=ls, leaf_logp=pS, dleaf_logp=dc["dleaf"], d_rhs=d_rhs)
        dv, *l_aw = wave_backward(Pi, Pibar, row_max, ws, W, dts_r, c_out[0], consts, col_logp, tree,
                                  neumann_terms=int(so["neumann_terms"]), leaf_state=ls, leaf_logp=pS, active=act,
                                  grad_col=d_gcol)
        aw = [(c_out[1 + k] + l_aw[k]).astype(F32) for k in range(6)]
        d_gpD += aw[0].sum(0, dtype=F32)
        d_gpS += aw[3].sum(0, dtype=F32)
        d_gE += (aw[0] + aw[2]).sum(0, dtype=F32)
        d_gEbar += aw[1].sum(0, dtype=F32)
        d_gEs1 += aw[5].sum(0, dtype=F32)
        d_gEs2 += aw[4].sum(0, dtype=F32)
        d_gmc += aw[2].sum(0, dtype=F32)
        if dts_r is not None:
            ud, A, side = dts_cross_backward(Pi, Pibar, dv, ws, meta, pD, pS, tree, d_rhs, active=act,
                                             grad_log_pD=d_gpD, grad_log_pS=d_gpS, grad_mt=d_gmc, mt=mc,
                                             row_max_all=row_max)
            pibar_vjp_tree(Pi, col_logp, ud, A, side, meta, tree, d_rhs, active=act, row_max_all=row_max,
                           grad_col=d_gcol)
            dts_backward_so(Pi, dPi, Pibar, dPibar, v_k, ws, meta, pD, pS, dc["dpd_param"], dc["dps_param"], mc,
                            dc["dMC"], row_max, tree, d_rhs, d_gpD, d_gpS, d_gmc, d_gcol)
    # ---- E side ----
    dE, dE_s1, dE_s2, dEbar = raw["dE"], raw["dE_s1"], raw["dE_s2"], raw["dEbar"]
    dpS, dpD, dpL = raw["dlog_pS"], raw["dlog_pD"], raw["dlog_pL"]
    E_new_r, Es1_r, Es2_r, Ebar_r, _ = e_step_forward(E, pS, pD, pL, mc, col_logp, tree)
    zeros = z()

    def vjp_E(g_new, g1, g2, gb):
        return e_step_vjp(E, E_new_r, Es1_r, Es2_r, Ebar_r, pS, pD, pL, col_logp, tree, g_new, g1, g2, gb)

    def so_E(g_new, g_ebar):  # x = (E*, E* as E_new, E_s1, E_s2, Ebar, ...), dE_new = dE
        return e_step_backward_so(E, E, E_s1, E_s2, Ebar, pS, pD, pL, tree, g_new, g_ebar, dE, dE, dE_s1, dE_s2,
                                  dEbar, dpS, dpD, dpL)

    n_fam = int(roots.shape[0])
    fam = F32(1.0) if n_fam == 1 else F32(n_fam)
    aux_lin = vjp_E(zeros, d_gEs1, d_gEs2, d_gEbar)[0]
    so_aux = so_E(zeros, acc["Ebar"])
    e2E = _exp2(E)
    norm = max(F32(1.0) - F32(e2E.mean(dtype=F32)), F32(np.finfo(np.float32).tiny))
    dnorm = F32(-_L * (e2E * dE).mean(dtype=F32))
    dg_norm = (fam * (-_L * e2E * dE / (F32(S) * norm) + e2E * dnorm / (F32(S) * norm * norm))).astype(F32)
    dq_E = (d_gE + aux_lin + so_aux[0] + dg_norm).astype(F32)
    so_w = so_E(wE, zeros)
    rhs_E = (dq_E + so_w[0]).astype(F32)

    def AG(w):
        return (w - vjp_E(w, zeros, zeros, zeros)[0]).astype(F32)

    dwE = bicgstab(AG, rhs_E, max_iter=so.get("bicgstab_max_iter", 500), tol=so.get("bicgstab_tol", 1e-7),
                   breakdown_tol=so.get("bicgstab_breakdown_tol", 1e-30))
    lin_p = vjp_E(dwE, zeros, zeros, d_gEbar)[1:]
    so_p = so_E(wE, acc["Ebar"])
    d_cot = ((d_gpS + lin_p[0] + so_p[1]).astype(F32), (d_gpD + lin_p[1] + so_p[2]).astype(F32),
             (lin_p[2] + so_p[3]).astype(F32), (d_gmc + lin_p[3] + so_p[4]).astype(F32),
             (d_gcol + lin_p[4] + so_p[5]).astype(F32))
    if debug_out is not None:
        debug_out.update(d_gE=d_gE, d_gpD=d_gpD, d_gpS=d_gpS, d_gmc=d_gmc, d_gEbar=d_gEbar, d_gEs1=d_gEs1,
                         d_gEs2=d_gEs2, dq_E=dq_E, dwE=dwE)
    # ---- smooth head: primal cotangents (hvp_exact.py:160-166) for the second-order term, the
    # tangent cotangents through the extraction's VJP ----
    base_p = vjp_E(wE, zeros, zeros, acc["Ebar"])[1:]
    cot = ((acc["pS"] + base_p[0]).astype(F32), (acc["pD"] + base_p[1]).astype(F32), base_p[2],
           (acc["mt"] + base_p[3]).astype(F32))
    lin_theta, _ = extract_parameters_vjp(theta, col_weights if col_weights is not None else np.zeros(S, F32), tree,
                                          *d_cot, uniform_fast=True)
    out = lin_theta.astype(np.float64) + head_hvp(theta, u, cot)
    return out.astype(F32).reshape(-1)
