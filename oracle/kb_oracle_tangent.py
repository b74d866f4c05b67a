"""CPU oracle for the forward-mode tangent (JVP) of the solver -- TEST INFRASTRUCTURE ONLY.

A numpy float32 restatement of the reference's tangent pass (the "tangent" benchmark config):
``newton/forward_tangent.py:29-215`` (``param_jvp_uniform``, ``_wave_tangent_constants``,
``jvp_root_scores`` with the fixed-count fused self-loop), ``kbench/core/kernels/e_step_tangent.py``
(``_e_step_tangent_2d_kernel`` :23-150, ``e_tangent_fixed_point`` :174-208),
``kbench/core/kernels/dts_tangent.py:23-122`` and ``kbench/core/kernels/wave_tangent.py:186-390``
(``_wave_step_tangent_selfloop_kernel``).  Only ``tests/`` may import it; the CUDA path never
calls into this file.  Pinned by ``tests/golden/make_golden.py`` (tangent cases run the reference
itself under ``TRITON_INTERPRET=1``).
"""

from __future__ import annotations

import numpy as np

from .kb_oracle import F32, NEG_INF, Tree, _f, _safe, dts_forward


def param_jvp_uniform(theta, v):
    """``forward_tangent.py:29-40``: tangent of ``extract_parameters_uniform`` along ``v``.
    With logits ``[0, theta]`` and ``p = softmax2(logits)``, ``d log2softmax_j = dl_j - sum_k p_k
    dl_k``; returns (dlog_pS, dlog_pD, dlog_pL, dmax_coupling)."""
    theta = np.asarray(theta, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    S = theta.shape[0]
    logits = np.concatenate([np.zeros((S, 1)), theta], axis=1)
    p = np.exp2(logits - logits.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    dl = np.concatenate([np.zeros((S, 1)), v], axis=1)
    dr = dl - (p * dl).sum(axis=1, keepdims=True)
    return tuple(dr[:, j].astype(F32) for j in range(4))


def e_step_tangent(E, dE, pS, pD, pL, mc, dpS, dpD, dpL, dmc, tree: Tree):
    """``e_step_tangent.py:23-150``: one linearised E application at the frozen E.
    Returns (dE_new, dE_s1, dE_s2, dEbar, max|dE_new - dE|)."""
    E, dE = _f(E), _f(dE)
    S = tree.S
    row_max = E.max()
    rms = F32(0.0) if row_max == NEG_INF else row_max
    r = np.exp2(E - rms).astype(F32)
    row_sum = r.sum(dtype=F32)
    dRS = (r * dE).sum(dtype=F32)
    anc = tree.ancestor_sum(r)
    dAS = tree.ancestor_sum((r * dE).astype(F32))
    E_s1 = tree.gather_child(E, 1)
    E_s2 = tree.gather_child(E, 2)
    dE_s1 = np.where(tree.c1_valid, dE[tree.c1_safe], F32(0.0)).astype(F32)
    dE_s2 = np.where(tree.c2_valid, dE[tree.c2_safe], F32(0.0)).astype(F32)
    denom = (row_sum - anc).astype(F32)
    pos = denom > 0
    sd = np.where(pos, denom, F32(1.0)).astype(F32)
    Ebar = np.where(pos, np.log2(sd) + row_max + _f(mc), NEG_INF).astype(F32)
    dEbar = np.where(pos, (dRS - dAS) / sd + _f(dmc), F32(0.0)).astype(F32)
    t0 = (_f(pS) + E_s1 + E_s2).astype(F32)
    t1 = (_f(pD) + F32(2.0) * E).astype(F32)
    t2 = (E + Ebar).astype(F32)
    t3 = _f(pL)
    m = np.maximum(np.maximum(t0, t1), np.maximum(t2, t3))
    ms = _safe(m)
    e = [np.exp2(t - ms).astype(F32) for t in (t0, t1, t2, t3)]
    total = (e[0] + e[1] + e[2] + e[3]).astype(F32)
    with np.errstate(divide="ignore"):
        E_new = (np.log2(total) + m).astype(F32)
    inv = np.where(total > 0, F32(1.0) / np.where(total > 0, total, F32(1.0)), F32(0.0)).astype(F32)
    dt = [(_f(dpS) + dE_s1 + dE_s2).astype(F32), (_f(dpD) + F32(2.0) * dE).astype(F32),
          (dE + dEbar).astype(F32), _f(dpL)]
    dE_new = sum((e[k] * inv) * dt[k] for k in range(4)).astype(F32)
    dE_new = np.where(E_new != NEG_INF, dE_new, F32(0.0)).astype(F32)
    return dE_new, dE_s1, dE_s2, dEbar, float(np.max(np.abs(dE_new - dE)))


def e_tangent_fixed_point(E_star, dpS, dpD, dpL, dmc, pS, pD, pL, mc, tree: Tree, *, max_iter, tol):
    """``e_step_tangent.py:174-208``: Richardson iteration from dE = 0 until
    ``max|dE_new - dE| <= tol * max(1, max|dE_new|)``, then one more application for
    (dE_s1, dE_s2, dEbar) at the final dE.  Returns (dE, dE_s1, dE_s2, dEbar, iterations)."""
    dE = np.zeros(tree.S, dtype=F32)
    n = 0
    for _ in range(int(max_iter)):
        dE_new, _, _, _, md = e_step_tangent(E_star, dE, pS, pD, pL, mc, dpS, dpD, dpL, dmc, tree)
        dE = dE_new
        n += 1
        if md <= tol * max(1.0, float(np.max(np.abs(dE)))):
            break
    _, dE_s1, dE_s2, dEbar, _ = e_step_tangent(E_star, dE, pS, pD, pL, mc, dpS, dpD, dpL, dmc, tree)
    return dE, dE_s1, dE_s2, dEbar, n


def tangent_constants(theta, v, saved, tree: Tree, *, e_max_iter, e_tol):
    """``forward_tangent.py:68-100`` ``_wave_tangent_constants``: parameter and E tangents
    assembled into the wave-step tangent constants (single item row)."""
    dpS, dpD, dpL, dmc = param_jvp_uniform(theta, v)
    dE, dE_s1, dE_s2, dEbar, n = e_tangent_fixed_point(
        saved["E"], dpS, dpD, dpL, dmc, saved["log_pS"], saved["log_pD"], saved["log_pL"],
        saved["max_coupling"], tree, max_iter=e_max_iter, tol=e_tol)
    return {
        "dDL": (dpD + dE).astype(F32), "dEbar": dEbar, "dE": dE, "dSL1": (dpS + dE_s2).astype(F32),
        "dSL2": (dpS + dE_s1).astype(F32), "dMC": dmc, "dleaf": dpS, "dpd_param": dpD, "dps_param": dpS,
        "raw": {"dlog_pS": dpS, "dlog_pD": dpD, "dlog_pL": dpL, "dmax_coupling": dmc, "dE": dE,
                "dE_s1": dE_s1, "dE_s2": dE_s2, "dEbar": dEbar, "e_iters": n},
    }


def dts_tangent(Pi, Pibar, dPi, dPibar, meta, pD, pS, dpD, dpS, dts_r, tree: Tree):
    """``dts_tangent.py:23-122``: ``d_dts[p,s] = sum over p's splits of sum_k 2^(t_k - dts_r[p,s])
    dt_k`` (zero where dts_r is -inf)."""
    W = int(meta["W"])
    S = tree.S
    sl = np.asarray(meta["sl"], dtype=np.int64)
    sr = np.asarray(meta["sr"], dtype=np.int64)
    red = np.asarray(meta["reduce_idx"], dtype=np.int64)
    lsp = meta.get("log_split_probs")
    lsp = np.zeros(sl.shape[0], F32) if lsp is None else _f(lsp).reshape(-1)
    out = np.zeros((W, S), dtype=F32)
    dts_r = _f(dts_r)
    for n in range(sl.shape[0]):
        l, r, p = sl[n], sr[n], red[n]
        pil, pir, pbl, pbr = Pi[l], Pi[r], Pibar[l], Pibar[r]
        dpl, dpr, dbl, dbr = dPi[l], dPi[r], dPibar[l], dPibar[r]
        t = [
            (lsp[n] + _f(pD) + pil + pir).astype(F32),
            (lsp[n] + pil + pbr).astype(F32),
            (lsp[n] + pir + pbl).astype(F32),
            (lsp[n] + _f(pS) + tree.gather_child(pil, 1) + tree.gather_child(pir, 2)).astype(F32),
            (lsp[n] + _f(pS) + tree.gather_child(pir, 1) + tree.gather_child(pil, 2)).astype(F32),
        ]

        def dg(x, which):
            v, idx = (tree.c1_valid, tree.c1_safe) if which == 1 else (tree.c2_valid, tree.c2_safe)
            return np.where(v, x[idx], F32(0.0)).astype(F32)

        dt = [
            (_f(dpD) + dpl + dpr).astype(F32), (dpl + dbr).astype(F32), (dpr + dbl).astype(F32),
            (_f(dpS) + dg(dpl, 1) + dg(dpr, 2)).astype(F32), (_f(dpS) + dg(dpr, 1) + dg(dpl, 2)).astype(F32),
        ]
        d = dts_r[p]
        contrib = sum(np.exp2(t[k] - d).astype(F32) * dt[k] for k in range(5)).astype(F32)
        out[p] = (out[p] + np.where(d != NEG_INF, contrib, F32(0.0))).astype(F32)
    return out


def wave_tangent_selfloop(pi_rows, dpi_rows, consts, dc, tree: Tree, n_iters, *, dts_r=None, d_dts=None,
                          leaf_state=None, leaf_logp=None):
    """``wave_tangent.py:186-336`` ``_wave_step_tangent_selfloop_kernel``: ``n_iters`` in-place
    Jacobi steps of the linearised wave step at the frozen primal rows.  Returns (dpi, dpibar of
    the last step)."""
    pi = _f(pi_rows)
    W, S = pi.shape
    row_max = pi.max(axis=1, keepdims=True)
    rms = _safe(row_max)
    r = np.exp2(pi - rms).astype(F32)
    row_sum = r.sum(axis=1, keepdims=True, dtype=F32)
    anc = tree.ancestor_sum(r)
    denom = (row_sum - anc).astype(F32)
    pos = denom > 0
    sd = np.where(pos, denom, F32(1.0)).astype(F32)
    inv_denom = np.where(pos, F32(1.0) / sd, F32(0.0)).astype(F32)
    pibar = np.where(pos, np.log2(sd) + row_max + _f(consts["mc"]), NEG_INF).astype(F32)
    t = [
        (_f(consts["dl"]) + pi).astype(F32), (pi + _f(consts["ebar"])).astype(F32),
        (pibar + _f(consts["e"])).astype(F32),
        (_f(consts["sl1"]) + tree.gather_child(pi, 1)).astype(F32),
        (_f(consts["sl2"]) + tree.gather_child(pi, 2)).astype(F32),
    ]
    t5 = np.full((W, S), NEG_INF, dtype=F32)
    dt5 = np.zeros((W, S), dtype=F32)
    if leaf_state is not None:
        rows = np.nonzero(leaf_state >= 0)[0]
        t5[rows, leaf_state[rows]] = _f(leaf_logp)[leaf_state[rows]]
        dt5[rows, leaf_state[rows]] = _f(dc["dleaf"])[leaf_state[rows]]
    t.append(t5)
    m = t[0]
    for x in t[1:]:
        m = np.maximum(m, x)
    if dts_r is not None:
        m = np.maximum(m, _f(dts_r))
    ms = _safe(m)
    e = [np.exp2(x - ms).astype(F32) for x in t]
    total = sum(e).astype(F32)
    num_dts = np.zeros((W, S), dtype=F32)
    if dts_r is not None:
        edts = np.exp2(_f(dts_r) - ms).astype(F32)
        total = (total + edts).astype(F32)
        num_dts = (edts * _f(d_dts)).astype(F32)
    with np.errstate(divide="ignore"):
        result = (np.log2(total) + m).astype(F32)
    inv = np.where(total > 0, F32(1.0) / np.where(total > 0, total, F32(1.0)), F32(0.0)).astype(F32)
    valid = result != NEG_INF
    dpi = _f(dpi_rows).copy()
    dpibar = np.zeros((W, S), dtype=F32)
    for _ in range(max(int(n_iters), 1)):
        dRS = (r * dpi).sum(axis=1, keepdims=True, dtype=F32)
        dAS = tree.ancestor_sum((r * dpi).astype(F32))
        dpibar = np.where(pos, (dRS - dAS) * inv_denom + _f(dc["dMC"]), F32(0.0)).astype(F32)
        d1 = np.where(tree.c1_valid, dpi[:, tree.c1_safe], F32(0.0)).astype(F32)
        d2 = np.where(tree.c2_valid, dpi[:, tree.c2_safe], F32(0.0)).astype(F32)
        dt = [(_f(dc["dDL"]) + dpi).astype(F32), (dpi + _f(dc["dEbar"])).astype(F32),
              (dpibar + _f(dc["dE"])).astype(F32), (_f(dc["dSL1"]) + d1).astype(F32),
              (_f(dc["dSL2"]) + d2).astype(F32), dt5]
        num = (sum(e[k] * dt[k] for k in range(6)) + num_dts).astype(F32)
        dpi = np.where(valid, num * inv, F32(0.0)).astype(F32)
    return dpi, dpibar


def jvp_root_scores(static: dict, theta, v, saved: dict, *, self_iters):
    """``forward_tangent.py:105-215`` with ``self_iters`` (the fused fixed-count self-loop):
    ``d(Pi_root)/dtheta . v``.  Returns (root tangents [n_roots, S], dPi [C,S], dPibar [C,S],
    tangent constants)."""
    sh, wl, so = static["state_helpers"], static["wave_layout"], static["solver_options"]
    tree = Tree(sh)
    S = tree.S
    pi, pibar = _f(saved["pi_wave"]), _f(saved["pibar_wave"])
    E, Ebar = _f(saved["E"]).reshape(-1), _f(saved["Ebar"]).reshape(-1)
    E_s1, E_s2 = _f(saved["E_s1"]).reshape(-1), _f(saved["E_s2"]).reshape(-1)
    pS, pD = _f(saved["log_pS"]).reshape(-1), _f(saved["log_pD"]).reshape(-1)
    mc = _f(saved["max_coupling"]).reshape(-1)
    consts = {"dl": (F32(1.0) + pD + E).astype(F32), "ebar": Ebar, "e": E,
              "sl1": (pS + E_s2).astype(F32), "sl2": (pS + E_s1).astype(F32), "mc": mc}
    dc = tangent_constants(theta, v, {k: _f(saved[k]).reshape(-1) for k in
                                      ("E", "log_pS", "log_pD", "log_pL", "max_coupling")},
                           tree, e_max_iter=so["e_max_iter"], e_tol=so.get("tangent_e_tol", 1e-6))
    C = pi.shape[0]
    dpi = np.zeros((C, S), dtype=F32)
    dpibar = np.zeros((C, S), dtype=F32)
    leaf_state_all = np.asarray(wl["leaf_state_index"], dtype=np.int64)
    for meta in wl["wave_metas"]:
        ws, W = int(meta["start"]), int(meta["W"])
        has_splits = "sl" in meta
        if has_splits:
            dts_r = dts_forward(pi, pibar, meta, pD, pS, tree)
            d_dts = dts_tangent(pi, pibar, dpi, dpibar, meta, pD, pS, dc["dpd_param"], dc["dps_param"], dts_r,
                                tree)
            ls = None
        else:
            dts_r = d_dts = None
            ls = leaf_state_all[ws:ws + W]
        dpi[ws:ws + W], dpibar[ws:ws + W] = wave_tangent_selfloop(
            pi[ws:ws + W], dpi[ws:ws + W], consts, dc, tree, self_iters, dts_r=dts_r, d_dts=d_dts,
            leaf_state=ls, leaf_logp=pS)
    roots = np.asarray(wl["root_row_ids"], dtype=np.int64)
    return dpi[roots], dpi, dpibar, dc
