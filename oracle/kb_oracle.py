"""CPU oracle for the solver hot path -- TEST INFRASTRUCTURE ONLY.

This module is a plain numpy (float32) restatement of the reference's numerics for the hot path:
the E-step fixed point and its VJP, the split reduction (``dts``), the wave fixed-point sweep,
the implicit adjoint with its parameter VJP, the E-adjoint BiCGSTAB solve and the theta VJP.
It follows the *pristine* reference kernels (the golden producer of the reference project) and
the reference's orchestration glue; every function cites the file:line it restates (paths are
relative to the reference project root).

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg / ``--impl reference`` arm of ``bench.py`` may import it.  The CUDA path in
``kernel-bench_b200/kbench_b200`` never calls into this file.

Parity pin: ``tests/golden/make_golden.py`` runs the reference itself (its pristine Triton
kernels under ``TRITON_INTERPRET=1`` on the CPU) on generated problems and stores the results in
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this oracle against them.
"""

from __future__ import annotations

import math
import types
from pathlib import Path

import numpy as np

F32 = np.float32
NEG_INF = F32(-np.inf)
LN2 = 0.6931471805599453


def at_precision(dtype) -> types.ModuleType:
    """A fresh copy of this module whose arithmetic type is ``dtype`` (e.g. ``numpy.float64``).

    Every array, constant and default argument of the copy is built from its module-level ``F32``,
    so the copy evaluates the same algorithm (same operations in the same order, same stopping
    rules) at the higher precision: the yardstick for how far fp32 implementations of it -- the
    reference's and ours -- are from the algorithm's exact value."""
    name = np.dtype(dtype).name
    src = Path(__file__).read_text()
    anchor = "\nF32 = np.float32\n"
    if anchor not in src:
        raise RuntimeError("kb_oracle: dtype anchor not found")
    mod = types.ModuleType(f"kb_oracle_{name}")
    mod.__file__ = __file__
    exec(compile(src.replace(anchor, f"\nF32 = np.{name}\n", 1), __file__, "exec"), mod.__dict__)
    return mod


def _f(x):
    return np.asarray(x, dtype=F32)


def _safe(m):
    """Replace -inf by 0 (the ``m_safe`` idiom of every LSE in the reference kernels)."""
    return np.where(m == NEG_INF, F32(0.0), m).astype(F32)


def _lse_terms(terms):
    """max-then-sum log2-sum-exp2 over a list of same-shape float32 arrays."""
    m = terms[0]
    for t in terms[1:]:
        m = np.maximum(m, t)
    ms = _safe(m)
    s = np.zeros_like(m, dtype=F32)
    for t in terms:
        s = s + np.exp2(t - ms).astype(F32)
    with np.errstate(divide="ignore"):
        return (np.log2(s) + m).astype(F32)


class Tree:
    """Species-tree helpers (``state_helpers`` of the static layout)."""

    def __init__(self, sh: dict):
        self.S = int(sh["S"])
        S = self.S
        self.parent = np.asarray(sh["node_parent"], dtype=np.int64)
        self.c1 = np.asarray(sh["node_child1"], dtype=np.int64)
        self.c2 = np.asarray(sh["node_child2"], dtype=np.int64)
        self.sub_start = np.asarray(sh["node_subtree_start"], dtype=np.int64)
        self.sub_end = np.asarray(sh["node_subtree_end"], dtype=np.int64)
        self.max_depth = max(1, int(sh["max_ancestor_depth"]))
        self.unnorm_row_max = _f(sh["unnorm_row_max"])
        self.lv_ptr = np.asarray(sh["compact_level_ptr"], dtype=np.int64)
        self.lv_par = np.asarray(sh["compact_level_parents"], dtype=np.int64)
        self.lv_c1 = np.asarray(sh["compact_level_child1"], dtype=np.int64)
        self.lv_c2 = np.asarray(sh["compact_level_child2"], dtype=np.int64)
        self.c1_valid = (self.c1 >= 0) & (self.c1 < S)
        self.c2_valid = (self.c2 >= 0) & (self.c2 < S)
        self.c1_safe = np.where(self.c1_valid, self.c1, 0)
        self.c2_safe = np.where(self.c2_valid, self.c2, 0)

    def ancestor_sum(self, vals):
        """sum over ancestors-or-self of ``vals[..., s]``, accumulated self first, then parent,
        grandparent ... for ``max_ancestor_depth`` steps (``experiments/pristine_kernels/
        wave_step.py:62-89`` ``_pibar_tile``; ``e_step.py:52-62``)."""
        S = self.S
        cur = np.arange(S)
        acc = np.zeros(vals.shape, dtype=F32)
        for _ in range(self.max_depth):
            valid = (cur >= 0) & (cur < S)
            if not valid.any():
                break
            safe = np.where(valid, cur, 0)
            acc = acc + np.where(valid, vals[..., safe], F32(0.0)).astype(F32)
            cur = np.where(valid, self.parent[safe], -1)
        return acc

    def subtree_sums_inplace(self, x):
        """Bottom-up subtree sums over compact levels, deepest level first, in place:
        ``x[p] = x[p] + x[c1] + x[c2]`` (``experiments/pristine_kernels/wave_backward.py:456-499``,
        ``:2396-2413``)."""
        S = self.S
        for lv in range(len(self.lv_ptr) - 1):
            a, b = self.lv_ptr[lv], self.lv_ptr[lv + 1]
            p = self.lv_par[a:b]
            c1 = self.lv_c1[a:b]
            c2 = self.lv_c2[a:b]
            v1 = np.where(c1 < S, x[..., np.where(c1 < S, c1, 0)], F32(0.0))
            v2 = np.where(c2 < S, x[..., np.where(c2 < S, c2, 0)], F32(0.0))
            x[..., p] = (x[..., p] + v1 + v2).astype(F32)
        return x

    def gather_child(self, rows, which):
        """rows[..., c(s)] with -inf where s has no such child."""
        if which == 1:
            return np.where(self.c1_valid, rows[..., self.c1_safe], NEG_INF).astype(F32)
        return np.where(self.c2_valid, rows[..., self.c2_safe], NEG_INF).astype(F32)


# ----------------------------------------------------------------------------------------------
# parameters  (kbench/core/parameters/extract_parameters.py)
# ----------------------------------------------------------------------------------------------

def extract_parameters_uniform(theta, unnorm_row_max):
    """``extract_parameters.py:25-34`` (statewise, not itemwise): log2-softmax of
    ``[0, theta0, theta1, theta2]`` -> (log_pS, log_pD, log_pL, max_coupling=log_pT+urm)."""
    theta = np.asarray(theta, dtype=np.float64)
    logits = np.concatenate([np.zeros((theta.shape[0], 1)), theta], axis=1)
    m = logits.max(axis=1, keepdims=True)
    lse = m + np.log2(np.exp2(logits - m).sum(axis=1, keepdims=True))
    r = (logits - lse).astype(F32)
    mc = (r[:, 3] + _f(unnorm_row_max)).astype(F32)
    return r[:, 0].copy(), r[:, 1].copy(), r[:, 2].copy(), mc


def col_weights_are_uniform(col_weights) -> bool:
    """``solver.py:11-13``: every entry equal (or no weights given)."""
    if col_weights is None:
        return True
    w = np.asarray(col_weights).reshape(-1)
    return bool(np.all(w == w[0]))


def extract_parameters_weighted(theta, col_weights, tree: Tree):
    """``extract_parameters.py:68-93`` (statewise, not itemwise, ``uniform_fast=False``) in fp32:
    col_log_probs = log_softmax(w) / ln 2 (``:37-38``), the column normaliser
    ``-log2(1 - ancestor-or-self mass)`` (``:41-65``, one ancestor per round, self first), and
    max_coupling = log_pT + normaliser.  Returns (log_pS, log_pD, log_pL, max_coupling, clp)."""
    S = tree.S
    pS, pD, pL, log_pT = extract_parameters_uniform(theta, np.zeros(S, F32))
    w = _f(col_weights).reshape(-1)
    m = w.max()
    lse = (m + np.log(np.exp(w - m, dtype=F32).sum(dtype=F32))).astype(F32)
    clp = ((w - lse) / F32(LN2)).astype(F32)
    col_p = np.exp2(clp).astype(F32)
    anc = np.zeros(S, F32)
    cur = np.arange(S)
    for _ in range(tree.max_depth):
        valid = (cur >= 0) & (cur < S)
        safe = np.where(valid, cur, 0)
        anc = (anc + np.where(valid, col_p[safe], F32(0.0))).astype(F32)
        cur = np.where(valid, tree.parent[safe], -1)
    vm = (F32(1.0) - anc).astype(F32)
    tiny = np.finfo(np.float32).tiny
    with np.errstate(divide="ignore"):
        norm = np.where(vm > 0.0, -np.log2(np.maximum(vm, tiny)), -np.inf).astype(F32)
    mc = (log_pT + norm).astype(F32)
    return pS, pD, pL, mc, clp


def extract_parameters_vjp(theta, col_weights, tree: Tree, g_pS, g_pD, g_pL, g_mt, g_col,
                           *, uniform_fast=True):
    """VJP of ``extract_parameters_weighted_cols`` (``extract_parameters.py:68-93``, with
    ``col_valid_log_normalizer`` ``:41-65`` and ``col_log_probs_from_weights`` ``:37-38``) from
    cotangents on (log_pS, log_pD, log_pL, max_coupling, col_log_probs) to (theta, col_weights).
    """
    theta = np.asarray(theta, dtype=np.float64)
    S = tree.S
    logits = np.concatenate([np.zeros((S, 1)), theta], axis=1)
    p = np.exp2(logits - logits.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    g = np.stack([g_pS, g_pD, g_pL, g_mt], axis=1).astype(np.float64)  # mt = log_pT + ...
    g_logits = g - p * g.sum(axis=1, keepdims=True)
    grad_theta = g_logits[:, 1:]
    # col_log_probs = log_softmax(w)/ln2 ; col_norm[s] = -log2(1 - sum_anc 2^clp)
    w = np.asarray(col_weights, dtype=np.float64)
    q = np.exp(w - w.max())
    q /= q.sum()
    clp = np.log(q) / LN2
    col_p = np.exp2(clp)
    anc_mass = np.zeros(S)
    cur = np.arange(S)
    for _ in range(tree.max_depth):
        valid = (cur >= 0) & (cur < S)
        safe = np.where(valid, cur, 0)
        anc_mass += np.where(valid, col_p[safe], 0.0)
        cur = np.where(valid, tree.parent[safe], -1)
    vm = 1.0 - anc_mass
    # d col_norm[s] / d clp[a] = 2^clp[a] / vm[s] for a anc-or-self of s
    coef = np.where(vm > 0, np.asarray(g_mt, dtype=np.float64) / np.maximum(vm, 1e-300), 0.0)
    # sum over s in subtree(a) of coef[s]  ->  bottom-up subtree sums
    sub = coef.copy()
    for lv in range(len(tree.lv_ptr) - 1):
        a, b = tree.lv_ptr[lv], tree.lv_ptr[lv + 1]
        pr = tree.lv_par[a:b]
        sub[pr] += np.where(tree.lv_c1[a:b] < S, sub[np.minimum(tree.lv_c1[a:b], S - 1)], 0.0) \
            + np.where(tree.lv_c2[a:b] < S, sub[np.minimum(tree.lv_c2[a:b], S - 1)], 0.0)
    g_clp = np.asarray(g_col, dtype=np.float64) + col_p * sub
    g_w = (g_clp - q * g_clp.sum()) / LN2
    return grad_theta.astype(F32), g_w.astype(F32)


# ----------------------------------------------------------------------------------------------
# E-step  (kbench/core/kernels/e_step.py)
# ----------------------------------------------------------------------------------------------

def e_step_forward(E, pS, pD, pL, mc, col_logp, tree: Tree, use_col_weights=False):
    """One E application (``e_step.py:12-99`` ``_e_step_forward_2d_kernel``), E is ``[S]``.
    Returns (E_new, E_s1, E_s2, Ebar, max_diff)."""
    E = _f(E)
    weighted = (_f(col_logp) + E).astype(F32) if use_col_weights else E
    row_max = weighted.max()
    rms = F32(0.0) if row_max == NEG_INF else row_max
    ex = np.exp2(weighted - rms).astype(F32)
    row_sum = ex.sum(dtype=F32)
    anc = tree.ancestor_sum(ex)
    E_s1 = tree.gather_child(E, 1)
    E_s2 = tree.gather_child(E, 2)
    denom = (row_sum - anc).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        Ebar = np.where(denom > 0, np.log2(np.where(denom > 0, denom, 1)) + row_max + _f(mc),
                        NEG_INF).astype(F32)
    t0 = (_f(pS) + E_s1 + E_s2).astype(F32)
    t1 = (_f(pD) + F32(2.0) * E).astype(F32)
    t2 = (E + Ebar).astype(F32)
    t3 = _f(pL)
    E_new = _lse_terms([t0, t1, t2, t3])
    with np.errstate(invalid="ignore"):
        max_diff = float(np.max(np.abs(E_new - E)))
    return E_new, E_s1, E_s2, Ebar, max_diff


def e_fixed_point(E0, pS, pD, pL, mc, col_logp, tree, *, max_iter, tol, use_col_weights=False):
    """``e_step.py:438-501`` ``e_fixed_point_triton``: iterate until max|dE| < tol or max_iter,
    then one more application for (E_s1, E_s2, Ebar) at the final E. Returns also the count."""
    E = _f(E0).copy()
    n = 0
    for _ in range(int(max_iter)):
        E_new, _, _, _, md = e_step_forward(E, pS, pD, pL, mc, col_logp, tree, use_col_weights)
        E = E_new
        n += 1
        if md < tol:
            break
    _, E_s1, E_s2, Ebar, _ = e_step_forward(E, pS, pD, pL, mc, col_logp, tree, use_col_weights)
    return E, E_s1, E_s2, Ebar, n


def e_step_vjp(E, E_new, E_s1, E_s2, Ebar, pS, pD, pL, col_logp, tree: Tree,
               g_new, g_s1, g_s2, g_ebar, use_col_weights=False):
    """VJP of one E application (``e_step.py:102-241`` prepare + finalize, ``:325-409``).
    Returns (grad_E, grad_pS, grad_pD, grad_pL, grad_mc, grad_col)."""
    S = tree.S
    E = _f(E)
    weighted = (_f(col_logp) + E).astype(F32) if use_col_weights else E
    row_max = weighted.max()
    rms = F32(0.0) if row_max == NEG_INF else row_max
    r = np.exp2(weighted - rms).astype(F32)
    row_sum = r.sum(dtype=F32)
    t0 = (_f(pS) + _f(E_s1) + _f(E_s2)).astype(F32)
    t1 = (_f(pD) + F32(2.0) * E).astype(F32)
    t2 = (E + _f(Ebar)).astype(F32)
    t3 = _f(pL)
    En = _f(E_new)
    g_new = _f(g_new)
    q0 = (g_new * np.exp2(t0 - En)).astype(F32)
    q1 = (g_new * np.exp2(t1 - En)).astype(F32)
    q2 = (g_new * np.exp2(t2 - En)).astype(F32)
    q3 = (g_new * np.exp2(t3 - En)).astype(F32)
    wbar = (q2 + _f(g_ebar)).astype(F32)
    grad_E = (F32(2.0) * q1 + q2).astype(F32)
    np.add.at(grad_E, tree.c1[tree.c1_valid], (q0 + _f(g_s1))[tree.c1_valid])
    np.add.at(grad_E, tree.c2[tree.c2_valid], (q0 + _f(g_s2))[tree.c2_valid])
    anc = tree.ancestor_sum(r)
    denom = (row_sum - anc).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        u = np.where(denom > 0, wbar / np.where(denom > 0, denom, 1), F32(0.0)).astype(F32)
    total_u = u.sum(dtype=F32)
    # excluded[x] = sum of u over s with x anc-or-self of s = subtree sum of u at x
    excluded = u.copy()
    tree.subtree_sums_inplace(excluded)
    pibar_vjp = (r * (total_u - excluded)).astype(F32)
    grad_E = (grad_E + pibar_vjp).astype(F32)
    grad_col = pibar_vjp.copy()
    return grad_E, q0, q1, q3, wbar, grad_col


# ----------------------------------------------------------------------------------------------
# split reduction  (kbench/core/kernels/dts_fused.py)
# ----------------------------------------------------------------------------------------------

def dts_split_terms(Pi, Pibar, l, r, lsp, log_pD, log_pS, tree: Tree):
    """The five terms of one split (``dts_fused.py:54-60``): arrays [S]."""
    pi_l, pi_r, pb_l, pb_r = Pi[l], Pi[r], Pibar[l], Pibar[r]
    lsp = F32(lsp)
    t0 = (lsp + _f(log_pD) + pi_l + pi_r).astype(F32)
    t1 = (lsp + pi_l + pb_r).astype(F32)
    t2 = (lsp + pi_r + pb_l).astype(F32)
    t3 = (lsp + _f(log_pS) + tree.gather_child(pi_l, 1) + tree.gather_child(pi_r, 2)).astype(F32)
    t4 = (lsp + _f(log_pS) + tree.gather_child(pi_r, 1) + tree.gather_child(pi_l, 2)).astype(F32)
    return [t0, t1, t2, t3, t4]


def dts_forward(Pi, Pibar, meta: dict, log_pD, log_pS, tree: Tree, active=None):
    """``compute_dts_forward`` (``dts_fused.py:171-231``): per parent row, the log2-sum-exp2 of the
    five split terms over all of its splits; single-split parents in closed form (``:18-62``),
    multi-split parents by an online LSE over splits (``:65-168``); inactive parents -> -inf."""
    W = int(meta["W"])
    S = tree.S
    out = np.full((W, S), NEG_INF, dtype=F32)
    sl = np.asarray(meta["sl"]); sr = np.asarray(meta["sr"])
    red = np.asarray(meta["reduce_idx"]); lsp = np.asarray(meta["log_split_probs"], dtype=F32)
    n_eq1 = int(meta["n_eq1"])
    for n in range(n_eq1):
        w = int(red[n])
        if active is not None and not active[w]:
            continue
        out[w] = _lse_terms(dts_split_terms(Pi, Pibar, int(sl[n]), int(sr[n]), lsp[n],
                                            log_pD, log_pS, tree))
    ptr = np.asarray(meta["ge2_ptr"]); parents = np.asarray(meta["ge2_parent_ids"])
    for g in range(len(parents)):
        w = int(parents[g])
        if active is not None and not active[w]:
            continue
        m = np.full(S, NEG_INF, dtype=F32)
        acc = np.zeros(S, dtype=F32)
        for rel in range(int(ptr[g]), int(ptr[g + 1])):
            i = n_eq1 + rel
            terms = dts_split_terms(Pi, Pibar, int(sl[i]), int(sr[i]), lsp[i], log_pD, log_pS, tree)
            sm = terms[0]
            for t in terms[1:]:
                sm = np.maximum(sm, t)
            sms = _safe(sm)
            ssum = np.zeros(S, dtype=F32)
            for t in terms:
                ssum = ssum + np.exp2(t - sms).astype(F32)
            new_m = np.maximum(m, sm)
            nms = _safe(new_m)
            acc = (np.where(m != NEG_INF, acc * np.exp2(m - nms), F32(0.0))
                   + ssum * np.exp2(sms - nms)).astype(F32)
            m = new_m
        with np.errstate(divide="ignore"):
            out[w] = (np.log2(acc) + m).astype(F32)
    return out


# ----------------------------------------------------------------------------------------------
# wave forward  (kbench/core/kernels/wave_step.py, kbench/core/inference/forward.py)
# ----------------------------------------------------------------------------------------------

def pibar_rows(Pi_rows, mc, col_logp, tree: Tree, use_col_weights=False):
    """Pibar from a block of Pi rows (``experiments/pristine_kernels/wave_step.py:26-89``):
    ``log2(rowsum - ancestor-or-self sum of 2^(Pi-rowmax)) + rowmax + mc``.
    Returns (Pibar, row_max)."""
    weighted = (Pi_rows + _f(col_logp)).astype(F32) if use_col_weights else Pi_rows
    row_max = weighted.max(axis=-1)
    rms = _safe(row_max)
    ex = np.exp2(weighted - rms[:, None]).astype(F32)
    row_sum = ex.sum(axis=-1, dtype=F32)
    anc = tree.ancestor_sum(ex)
    denom = (row_sum[:, None] - anc).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        pib = np.where(denom > 0, np.log2(np.where(denom > 0, denom, 1)) + row_max[:, None]
                       + _f(mc), NEG_INF).astype(F32)
    return pib, row_max.astype(F32)


def wave_step(Pi_in_rows, consts: dict, col_logp, tree: Tree, *, leaf_state=None,
              leaf_logp=None, dts_r=None, use_col_weights=False):
    """One Jacobi sweep of a wave (``experiments/pristine_kernels/wave_step.py:92-220``):
    ``Pi_new = lse2(dl+Pi, Pi+ebar, Pibar+e, sl1+Pi[c1], sl2+Pi[c2], leaf, dts)``."""
    pi = _f(Pi_in_rows)
    pib, _ = pibar_rows(pi, consts["mc"], col_logp, tree, use_col_weights)
    terms = [
        (consts["dl"] + pi).astype(F32),
        (pi + consts["ebar"]).astype(F32),
        (pib + consts["e"]).astype(F32),
        (consts["sl1"] + tree.gather_child(pi, 1)).astype(F32),
        (consts["sl2"] + tree.gather_child(pi, 2)).astype(F32),
    ]
    if leaf_state is not None:
        t5 = np.full(pi.shape, NEG_INF, dtype=F32)
        rows = np.nonzero(leaf_state >= 0)[0]
        t5[rows, leaf_state[rows]] = _f(leaf_logp)[leaf_state[rows]]
        terms.append(t5)
    if dts_r is not None:
        terms.append(_f(dts_r))
    return _lse_terms(terms)


def leaf_initial(consts: dict, col_logp, tree: Tree, leaf_state, leaf_logp,
                 use_col_weights=False):
    """Leaf seed (``experiments/pristine_kernels/wave_step.py:223-310``): Pi is the leaf
    log-probability at the leaf column, Pibar is ``mc + col[leaf] + leaf_obs`` outside the leaf's
    subtree; one LSE step."""
    W = leaf_state.shape[0]
    S = tree.S
    cols = np.arange(S)
    leaf_logp = _f(leaf_logp)
    out = np.empty((W, S), dtype=F32)
    for w in range(W):
        ls = int(leaf_state[w])
        obs = leaf_logp[ls]
        desc = (tree.sub_start >= tree.sub_start[ls]) & (tree.sub_start < tree.sub_end[ls])
        hit = cols == ls
        colp = _f(col_logp)[ls] if use_col_weights else F32(0.0)
        pi_w = np.where(hit, obs, NEG_INF).astype(F32)
        pib = np.where(~desc, (consts["mc"] + colp + obs).astype(F32), NEG_INF).astype(F32)
        ps1 = np.where(tree.c1 == ls, obs, NEG_INF).astype(F32)
        ps2 = np.where(tree.c2 == ls, obs, NEG_INF).astype(F32)
        t5 = np.where(hit, leaf_logp, NEG_INF).astype(F32)
        out[w] = _lse_terms([
            (consts["dl"] + pi_w).astype(F32), (pi_w + consts["ebar"]).astype(F32),
            (pib + consts["e"]).astype(F32), (consts["sl1"] + ps1).astype(F32),
            (consts["sl2"] + ps2).astype(F32), t5,
        ])
    return out


def forward(static: dict, theta, col_weights=None, *, pi_iters=None, e_init=None):
    """theta -> (loss, saved): ``kbench/runtime.py:63-74`` -> ``solver.py:16-96`` (E fixed point,
    ``forward.py:8-117`` wave loop) -> ``solver.py:132-142`` NLL; non-uniform ``col_weights``
    take the weighted-column parameters and kernels (``use_col_weights``) as the reference does."""
    sh = static["state_helpers"]
    wl = static["wave_layout"]
    so = static["solver_options"]
    tree = Tree(sh)
    S = tree.S
    ucw = not col_weights_are_uniform(col_weights)  # solver.py:27-44
    if ucw:
        pS, pD, pL, mc, col_logp = extract_parameters_weighted(theta, col_weights, tree)
    else:
        pS, pD, pL, mc = extract_parameters_uniform(theta, sh["unnorm_row_max"])
        col_logp = np.full(S, -math.log2(S), dtype=F32)
    E0 = np.full(S, float(so.get("e_init", -1.0) if e_init is None else e_init), dtype=F32)
    E, E_s1, E_s2, Ebar, n_e = e_fixed_point(E0, pS, pD, pL, mc, col_logp, tree,
                                             max_iter=so["e_max_iter"], tol=so["e_tol"],
                                             use_col_weights=ucw)
    pi_iters = int(so["pi_iters"] if pi_iters is None else pi_iters)
    consts = {
        "dl": (F32(1.0) + pD + E).astype(F32), "ebar": Ebar, "e": E,
        "sl1": (pS + E_s2).astype(F32), "sl2": (pS + E_s1).astype(F32), "mc": mc,
    }
    leaf_state_all = np.asarray(wl["leaf_state_index"], dtype=np.int64)
    C = leaf_state_all.shape[0]
    pi = np.full((C, S), np.nan, dtype=F32)
    pibar = np.full((C, S), np.nan, dtype=F32)
    row_max = np.full(C, np.nan, dtype=F32)
    for meta in wl["wave_metas"]:
        ws, W = int(meta["start"]), int(meta["W"])
        has_leaf = "sl" not in meta
        dts_r = None if has_leaf else dts_forward(pi, pibar, meta, pD, pS, tree)
        leaf_state = leaf_state_all[ws:ws + W] if has_leaf else None
        bufs = (pi, pibar)
        for it in range(pi_iters):
            pi_in, pi_out = (bufs[0], bufs[1]) if it % 2 == 0 else (bufs[1], bufs[0])
            if it == 0 and not has_leaf:
                continue
            if it == 0:
                pi_out[ws:ws + W] = leaf_initial(consts, col_logp, tree, leaf_state, pS, use_col_weights=ucw)
                continue
            src = dts_r if (it == 1 and not has_leaf) else pi_in[ws:ws + W]
            new = wave_step(src, consts, col_logp, tree, leaf_state=leaf_state, leaf_logp=pS,
                            dts_r=dts_r, use_col_weights=ucw)
            pi_out[ws:ws + W] = new
            if it == pi_iters - 1:
                pib, rmax = pibar_rows(new, mc, col_logp, tree, use_col_weights=ucw)
                pibar[ws:ws + W] = pib
                row_max[ws:ws + W] = rmax
    roots = np.asarray(wl["root_row_ids"], dtype=np.int64)
    loss = nll(pi[roots], E)
    saved = {"E": E, "E_s1": E_s1, "E_s2": E_s2, "Ebar": Ebar, "root_rows": pi[roots],
             "pi_wave": pi, "pibar_wave": pibar, "pibar_row_max": row_max, "log_pS": pS,
             "log_pD": pD, "log_pL": pL, "max_coupling": mc, "col_log_probs": col_logp,
             "e_iters": n_e}
    return loss, saved


def lse_rows(x):
    """``logspace.py:12-16`` logsumexp2 over the last axis."""
    x = _f(x)
    m = x.max(axis=-1, keepdims=True)
    ms = np.where(m == NEG_INF, F32(0.0), m)
    tot = np.exp2(x - ms).sum(axis=-1, keepdims=True, dtype=F32)
    with np.errstate(divide="ignore"):
        res = np.where(tot > 0, np.log2(np.where(tot > 0, tot, 1)), NEG_INF) + m
    return res[..., 0].astype(F32)


def nll(root_rows, E):
    """``solver.py:132-142``: ``-sum_roots[lse2(root) - log2 S - log2(1 - mean 2^E)]``."""
    S = root_rows.shape[-1]
    norm = max(F32(1.0) - F32(np.exp2(_f(E)).mean(dtype=F32)), np.finfo(np.float32).tiny)
    vec = -(lse_rows(root_rows) - F32(math.log2(S)) - F32(np.log2(F32(norm))))
    return float(vec.astype(F32).sum(dtype=F32))


# ----------------------------------------------------------------------------------------------
# backward  (kbench/core/kernels/wave_backward.py, kbench/api/_implicit_grad.py)
# ----------------------------------------------------------------------------------------------

def active_mask(rhs, threshold, use_pruning=True):
    """``experiments/pristine_kernels/wave_backward.py:166-201``: ``max|rhs| >= thr`` (``>`` when
    pruning is off)."""
    mx = np.abs(_f(rhs)).max(axis=-1) if rhs.shape[-1] else np.zeros(rhs.shape[0], F32)
    return (mx > threshold) if not use_pruning else (mx >= threshold)


def _self_loop_terms(Pi, Pibar, rows, consts, tree, leaf_state, leaf_logp, dts_r_rows):
    """Recompute the forward self-loop terms of converged rows (``wave_backward.py:282-354``
    precompute / ``:790-850`` param_store): returns (e[0..5], inv_sum, w_L)."""
    pi = Pi[rows]
    pib = Pibar[rows]
    t = [
        (consts["dl"] + pi).astype(F32), (pi + consts["ebar"]).astype(F32),
        (pib + consts["e"]).astype(F32), (consts["sl1"] + tree.gather_child(pi, 1)).astype(F32),
        (consts["sl2"] + tree.gather_child(pi, 2)).astype(F32),
    ]
    t5 = np.full(pi.shape, NEG_INF, dtype=F32)
    if leaf_state is not None:
        ok = np.nonzero(leaf_state >= 0)[0]
        t5[ok, leaf_state[ok]] = _f(leaf_logp)[leaf_state[ok]]
    t.append(t5)
    m = t[0]
    for x in t[1:]:
        m = np.maximum(m, x)
    ms = _safe(m)
    e = [np.exp2(x - ms).astype(F32) for x in t]
    ssum = e[0] + e[1] + e[2] + e[3] + e[4] + e[5]
    with np.errstate(divide="ignore"):
        inv_sum = np.where(ssum > 0, F32(1.0) / np.where(ssum > 0, ssum, 1), F32(0.0)).astype(F32)
    if dts_r_rows is not None:
        with np.errstate(divide="ignore", invalid="ignore"):
            dts_l = (np.log2(ssum) + m).astype(F32)
            pm = np.maximum(dts_l, dts_r_rows)
            pms = _safe(pm)
            pnew = (np.log2(np.exp2(dts_l - pms) + np.exp2(dts_r_rows - pms)) + pm).astype(F32)
            w_L = np.where(dts_l != NEG_INF, np.exp2(dts_l - pnew), F32(0.0)).astype(F32)
    else:
        w_L = np.ones(pi.shape, dtype=F32)
    return e, inv_sum, w_L


def gmres_fixed(apply_a, b, max_iter):
    """Unrestarted GMRES with a fixed number of Arnoldi steps (``kbench/core/kernels/
    wave_backward.py:831-912``, ``experiments/pristine_kernels/wave_backward.py:574-655``): the
    Krylov basis by classical Gram-Schmidt with one re-orthogonalisation pass, an early stop when
    the new vector's norm falls to ``eps * max(|b|, 1)``, and the least-squares solve of the
    Hessenberg system.  ``b`` is the whole wave as one vector."""
    m = int(max_iter)
    shape = b.shape
    b = _f(b).reshape(-1)
    if m < 1:
        return np.zeros(shape, F32)
    beta = F32(np.sqrt(np.dot(b, b)))
    if float(beta) == 0.0:
        return np.zeros(shape, F32)
    V = np.zeros((m + 1, b.size), F32)
    V[0] = b / beta
    H = np.zeros((m + 1, m), F32)
    g = np.zeros(m + 1, F32)
    g[0] = beta
    steps = m
    stop = F32(np.finfo(F32).eps) * max(beta, F32(1.0))
    for j in range(m):
        w = _f(apply_a(V[j].reshape(shape))).reshape(-1)
        Q = V[: j + 1]
        h1 = (Q @ w).astype(F32)
        w1 = (w - Q.T @ h1).astype(F32)
        h2 = (Q @ w1).astype(F32)
        w2 = (w1 - Q.T @ h2).astype(F32)
        H[: j + 1, j] = h1 + h2
        nrm = F32(np.sqrt(np.dot(w2, w2)))
        H[j + 1, j] = nrm
        if nrm <= stop:
            steps = j + 1
            break
        if j + 1 < m:
            V[j + 1] = w2 / max(nrm, F32(np.finfo(F32).tiny))
    y = np.linalg.lstsq(H[: steps + 1, :steps], g[: steps + 1], rcond=None)[0].astype(F32)
    return (V[:steps].T @ y).astype(F32).reshape(shape)


def wave_backward(Pi, Pibar, row_max_all, ws, W, dts_r, rhs, consts, col_logp, tree: Tree,
                  *, neumann_terms, leaf_state=None, leaf_logp=None, active=None,
                  grad_col=None, use_col_weights=False, self_loop_solver="neumann", last_out=None,
                  initial_v=None, grad_targets=None):
    """``wave_backward_uniform_fused`` (``experiments/pristine_kernels/wave_backward.py:
    1270-1736`` retained 2D path): precompute (``:203-417``), the self-loop adjoint -- Neumann
    ``v = sum_n (J^T)^n rhs`` (``:419-570``) or GMRES on ``(I - J^T) v = rhs`` over the wave's
    active rows (``:1136-1185``) --, column gradient (``:654-745``) and the parameter store
    (``:747-966``).  Returns (v_k, aw0, aw1, aw2, aw345, aw3, aw4); v_k rows of inactive rows are
    NaN in the Neumann solve (uninitialised in the reference), zero in the GMRES solve.
    ``last_out`` ([W], Neumann with at least one term) receives ``|last term| / |v|`` per row
    (zero on inactive rows; ``:1275-1292``).

    ``initial_v`` ([W,S], Neumann only; ``:1190-1230``): ``v = initial_v``, then ``neumann_terms``
    fixed-point updates ``v <- rhs + J^T v`` on the active rows (the JT kernel with
    FIXED_POINT_UPDATE, ``:420-655``); inactive rows keep ``initial_v``; no last increment
    (``:1275-1280``).  ``grad_targets`` = (grad_log_pD, grad_log_pS, grad_E, grad_Ebar, grad_E_s1,
    grad_E_s2, grad_mt, param_grad_vector) (``:1294-1314`` and the ACCUM_GRADS branch of the
    parameter store, ``:907-959``): the active rows' buckets are summed over rows and ADDED into
    those arrays (pD += aw0 and pS += aw345 per column, or -- without param_grad_vector -- each row's
    sum over columns; E += aw0 + aw2, Ebar += aw1, E_s1 += aw4, E_s2 += aw3, mt += aw2); the six
    buckets are then returned as None."""
    S = tree.S
    act = np.ones(W, dtype=bool) if active is None else np.asarray(active, dtype=bool)
    rows_l = np.nonzero(act)[0]
    rows = ws + rows_l
    v_k = np.full((W, S), np.nan, dtype=F32) if initial_v is None else _f(initial_v).copy()
    aw = [np.zeros((W, S), dtype=F32) for _ in range(7)]
    if rows_l.size == 0:
        return (v_k, *((None,) * 6 if grad_targets is not None else (aw[0], aw[1], aw[2], aw[3], aw[4], aw[5])))
    ls = None if leaf_state is None else leaf_state[rows_l]
    dts_rows = None if dts_r is None else dts_r[rows_l]
    e, inv_sum, w_L = _self_loop_terms(Pi, Pibar, rows, consts, tree, ls, leaf_logp, dts_rows)
    rmax = row_max_all[rows]
    rms = _safe(rmax)
    pi = Pi[rows]
    weighted = (pi + _f(col_logp)).astype(F32) if use_col_weights else pi
    p_prime = np.exp2(weighted - rms[:, None]).astype(F32)
    row_sum = p_prime.sum(axis=-1, dtype=F32)
    anc = tree.ancestor_sum(p_prime)
    denom = (row_sum[:, None] - anc).astype(F32)
    with np.errstate(divide="ignore"):
        inv_denom = np.where(denom > 0, F32(1.0) / np.where(denom > 0, denom, 1), F32(0.0))
    diag = (w_L * (e[0] + e[1]) * inv_sum).astype(F32)
    coeff = (w_L * e[2] * inv_sum * inv_denom).astype(F32)
    sl1w = (w_L * e[3] * inv_sum).astype(F32)
    sl2w = (w_L * e[4] * inv_sum).astype(F32)
    edge = np.zeros_like(diag)
    edge[:, tree.c1[tree.c1_valid]] = sl1w[:, tree.c1_valid]
    edge[:, tree.c2[tree.c2_valid]] = sl2w[:, tree.c2_valid]
    par = tree.parent
    par_ok = par >= 0
    par_safe = np.where(par_ok, par, 0)
    rhs_a = _f(rhs)[rows_l]

    def jt(term):
        u = (term * coeff).astype(F32)
        A = u.sum(axis=-1, dtype=F32)
        corr = tree.subtree_sums_inplace(u.copy())
        base = (term * diag + p_prime * (A[:, None] - corr)).astype(F32)
        return (base + np.where(par_ok, term[:, par_safe], F32(0.0)) * edge).astype(F32)

    if str(self_loop_solver).strip().lower() == "gmres":
        if initial_v is not None:
            raise ValueError("GMRES self-loop solve does not support initial_v")
        v = gmres_fixed(lambda x: (x - jt(x)).astype(F32), rhs_a, int(neumann_terms))
        v_k[:] = F32(0.0)
    elif initial_v is not None:
        v = _f(initial_v)[rows_l].copy()
        for _ in range(int(neumann_terms)):
            v = (rhs_a + jt(v)).astype(F32)
    else:
        v = rhs_a.copy()
        term = rhs_a
        for _ in range(int(neumann_terms)):
            res = jt(term)
            v = (v + res).astype(F32)
            term = res
        if last_out is not None and int(neumann_terms) > 0:
            last_out[:] = F32(0.0)
            num = np.sqrt((term.astype(np.float64) ** 2).sum(axis=-1))
            den = np.maximum(np.sqrt((v.astype(np.float64) ** 2).sum(axis=-1)), np.finfo(np.float32).tiny)
            last_out[rows_l] = (num / den).astype(F32)
    v_k[rows_l] = v
    if grad_col is not None:
        u = (v * coeff).astype(F32)
        A = u.sum(axis=-1, dtype=F32)
        corr = tree.subtree_sums_inplace(u.copy())
        contrib = (p_prime * (A[:, None] - corr)).astype(F32)
        grad_col += contrib.sum(axis=0, dtype=F32)
    alpha = (v * w_L).astype(F32)
    a = [(alpha * e[k] * inv_sum).astype(F32) for k in range(6)]
    aw[0][rows_l] = a[0]
    aw[1][rows_l] = a[1]
    aw[2][rows_l] = a[2]
    aw[3][rows_l] = (a[3] + a[4] + a[5]).astype(F32)
    aw[4][rows_l] = a[3]
    aw[5][rows_l] = a[4]
    if grad_targets is not None:
        g_pD, g_pS, g_E, g_Ebar, g_Es1, g_Es2, g_mt, vector = grad_targets
        col = [x.sum(axis=0, dtype=F32) for x in aw[:6]]  # active rows only: the others are zero
        if vector:
            g_pD += col[0]
            g_pS += col[3]
        else:
            g_pD += aw[0].sum(axis=1, dtype=F32).sum(dtype=F32)
            g_pS += aw[3].sum(axis=1, dtype=F32).sum(dtype=F32)
        g_E += (col[0] + col[2]).astype(F32)
        g_Ebar += col[1]
        g_Es1 += col[5]
        g_Es2 += col[4]
        g_mt += col[2]
        return (v_k, None, None, None, None, None, None)
    return (v_k, aw[0], aw[1], aw[2], aw[3], aw[4], aw[5])


def dts_cross_backward(Pi, Pibar, v_k, ws, meta, log_pD, log_pS, tree: Tree, acc_rhs, *,
                       active, grad_log_pD, grad_log_pS, grad_mt, mt, row_max_all, side_threshold=0.0):
    """``dts_cross_backward_accum_fused`` as the backward glue calls it
    (``experiments/pristine_kernels/wave_backward.py:1529-1945``; call flags at
    ``kbench/api/_implicit_grad.py:300-331``: merged S-term, parameter and mt reductions, staged
    Pibar u_d with side-active flags: with ``side_threshold`` > 0 a side is active when the sum
    of its |u_d| exceeds it (``:1776-1779, 1877-1884``), else when any u_d is nonzero). Mutates
    acc_rhs and the grads. Returns (pibar_ud [2N,S], pibar_A [2N], side_active [2N])."""
    S = tree.S
    sl = np.asarray(meta["sl"]); sr = np.asarray(meta["sr"])
    red = np.asarray(meta["reduce_idx"]); lsp = np.asarray(meta["log_split_probs"], dtype=F32)
    N = sl.shape[0]
    ud = np.full((2 * N, S), np.nan, dtype=F32)
    A = np.full(2 * N, np.nan, dtype=F32)
    side = np.zeros(2 * N, dtype=bool)
    for i in range(N):
        w = int(red[i])
        if not active[w]:
            continue
        l, r = int(sl[i]), int(sr[i])
        d = dts_split_terms(Pi, Pibar, l, r, F32(0.0), log_pD, log_pS, tree)
        ppar = Pi[ws + w]
        pv = ppar != NEG_INF
        vk = v_k[w]
        vd = [(vk * np.where(pv, np.exp2(F32(lsp[i]) + dk - ppar), F32(0.0))).astype(F32)
              for dk in d]
        acc_rhs[l] += (vd[0] + vd[1]).astype(F32)
        acc_rhs[r] += (vd[0] + vd[2]).astype(F32)
        fl = Pibar[l] != NEG_INF
        fr = Pibar[r] != NEG_INF
        inv_l = np.where(fl, np.exp2(row_max_all[l] + _f(mt) - Pibar[l]), F32(0.0)).astype(F32)
        inv_r = np.where(fr, np.exp2(row_max_all[r] + _f(mt) - Pibar[r]), F32(0.0)).astype(F32)
        ud_l = (vd[2] * inv_l).astype(F32)
        ud_r = (vd[1] * inv_r).astype(F32)
        ud[i] = ud_l
        ud[N + i] = ud_r
        A[i] = ud_l.sum(dtype=F32)
        A[N + i] = ud_r.sum(dtype=F32)
        if side_threshold > 0.0:
            side[i] = np.abs(ud_l).sum(dtype=F32) > F32(side_threshold)
            side[N + i] = np.abs(ud_r).sum(dtype=F32) > F32(side_threshold)
        else:
            side[i] = np.abs(ud_l).max() != 0
            side[N + i] = np.abs(ud_r).max() != 0
        grad_log_pD += vd[0]
        grad_log_pS += (vd[3] + vd[4]).astype(F32)
        grad_mt += (vd[1] + vd[2]).astype(F32)
        m1, m2 = tree.c1_valid, tree.c2_valid
        np.add.at(acc_rhs[l], tree.c1[m1], vd[3][m1])
        np.add.at(acc_rhs[r], tree.c1[m1], vd[4][m1])
        np.add.at(acc_rhs[r], tree.c2[m2], vd[3][m2])
        np.add.at(acc_rhs[l], tree.c2[m2], vd[4][m2])
    return ud, A, side


def pibar_vjp_tree(Pi, col_logp, ud, A, side, meta, tree: Tree, acc_rhs, *, active, row_max_all,
                   grad_col, use_col_weights=False):
    """``uniform_cross_pibar_vjp_tree_from_ud_fused`` (``experiments/pristine_kernels/
    wave_backward.py:2356-2446``): per active split side, in-place subtree sums of ``u_d``, then
    ``p'_child (A - subtree)`` into the child's adjoint row and the column gradient."""
    sl = np.asarray(meta["sl"]); sr = np.asarray(meta["sr"]); red = np.asarray(meta["reduce_idx"])
    N = sl.shape[0]
    for row in range(2 * N):
        if not side[row]:
            continue
        i = row if row < N else row - N
        if not active[int(red[i])]:
            continue
        child = int(sl[i] if row < N else sr[i])
        tree.subtree_sums_inplace(ud[row])
        rm = row_max_all[child]
        rms = F32(0.0) if rm == NEG_INF else rm
        w = (Pi[child] + _f(col_logp)).astype(F32) if use_col_weights else Pi[child]
        pp = np.exp2(w - rms).astype(F32)
        contrib = (pp * (A[row] - ud[row])).astype(F32)
        acc_rhs[child] += contrib
        grad_col += contrib


def _safe_exp2_ratio(a, b):
    neg = a == NEG_INF
    return np.where(neg, F32(0.0), np.exp2(np.where(neg, 0, a) - np.where(neg, 0, b))).astype(F32)


def bicgstab(Av, b, *, max_iter=500, tol=1e-7, breakdown_tol=1e-30):
    """``kbench/api/_implicit_grad.py:28-94`` (float32 vectors, same stopping rules)."""
    x = np.zeros_like(b)
    r = (b - Av(x)).astype(F32)
    bnorm = max(float(np.linalg.norm(b)), 1.0)
    rel = float(np.linalg.norm(r)) / bnorm
    if rel <= tol:
        return x
    r_hat = r.copy()
    rho_old = F32(1.0); alpha = F32(1.0); omega = F32(1.0)
    v = np.zeros_like(b); p = np.zeros_like(b)
    k = 0
    for k in range(1, int(max_iter) + 1):
        rho = F32(np.dot(r_hat, r))
        if abs(float(rho)) <= breakdown_tol:
            break
        beta = F32((rho / rho_old) * (alpha / omega))
        p = (r + beta * (p - omega * v)).astype(F32)
        v = Av(p)
        den = F32(np.dot(r_hat, v))
        if abs(float(den)) <= breakdown_tol:
            break
        alpha = F32(rho / den)
        s = (r - alpha * v).astype(F32)
        if float(np.linalg.norm(s)) / bnorm <= tol:
            return (x + alpha * p).astype(F32)
        t = Av(s)
        tt = F32(np.dot(t, t))
        if abs(float(tt)) <= breakdown_tol:
            break
        omega = F32(np.dot(t, s) / tt)
        x = (x + alpha * p + omega * s).astype(F32)
        r = (s - omega * t).astype(F32)
        rel = float(np.linalg.norm(r)) / bnorm
        if rel <= tol:
            return x
        if abs(float(omega)) <= breakdown_tol:
            break
        rho_old = rho
    raise RuntimeError(f"E-adjoint BiCGSTAB solve failed after {k} iterations "
                       f"(relative residual {rel:.3e})")


def backward(static: dict, theta, col_weights, saved: dict, acc_dtype=F32):
    """(forward intermediates) -> (grad_theta, grad_col): ``kbench/runtime.py:77-115`` ->
    ``kbench/api/_implicit_grad.py:98-370`` (reverse wave loop) and ``:373-475`` (E adjoint and
    theta VJP); ``use_col_weights`` = not uniform ``col_weights`` (``runtime.py:84``)."""
    acc = backward_accumulators(static, saved, acc_dtype,
                                use_col_weights=not col_weights_are_uniform(col_weights))
    n_fam = int(np.asarray(static["wave_layout"]["root_row_ids"]).shape[0])
    return e_adjoint_and_theta_vjp(static, theta, col_weights, saved, Tree(static["state_helpers"]),
                                   acc["E"], acc["Ebar"], acc["E_s1"], acc["E_s2"], acc["pD"], acc["pS"],
                                   acc["mt"], acc["col"], n_fam=n_fam)


def backward_accumulators(static: dict, saved: dict, acc_dtype=F32, cache: list | None = None,
                          use_col_weights: bool = False, relres: dict | None = None) -> dict:
    """The reverse wave loop of ``kbench/api/_implicit_grad.py:98-370`` alone: the fp32 column
    accumulators ``pD, pS, mt, E, Ebar, E_s1, E_s2, col`` (``:144-158``) that the E adjoint and
    theta VJP consume.

    ``acc_dtype=np.float64`` keeps every per-wave / per-split fp32 partial as the reference
    computes it but adds them into float64 running sums: the accumulation-exact evaluation of the
    same algorithm (the reference's fp32 running sums lose low-order bits of small contributions
    once the sums have grown).

    ``cache`` (a list) receives one dict per wave in the order processed (reverse wave order):
    ``ws, W, v`` (the adjoint rows, zero on inactive rows), ``dts_r, active, has_splits, meta``
    -- the point cache of the exact-Hessian HVP (``newton/ggn.py:152-162``).

    ``relres`` (a dict) receives the reference glue's ``collect_backward_relres`` diagnostics
    (``kbench/api/_implicit_grad.py:189-195, 263-288``): per family the largest
    ``|last Neumann term| / |v|`` (``relres``) and largest ``|v|`` (``vk_mag``) over active rows."""
    sh = static["state_helpers"]
    wl = static["wave_layout"]
    so = static["solver_options"]
    tree = Tree(sh)
    S = tree.S
    Pi = _f(saved["pi_wave"]); Pibar = _f(saved["pibar_wave"])
    E = _f(saved["E"]).reshape(-1); Ebar = _f(saved["Ebar"]).reshape(-1)
    E_s1 = _f(saved["E_s1"]).reshape(-1); E_s2 = _f(saved["E_s2"]).reshape(-1)
    pS = _f(saved["log_pS"]).reshape(-1); pD = _f(saved["log_pD"]).reshape(-1)
    pL = _f(saved["log_pL"]).reshape(-1); mc = _f(saved["max_coupling"]).reshape(-1)
    col_logp = _f(saved["col_log_probs"]).reshape(-1)
    row_max = _f(saved["pibar_row_max"])
    C = Pi.shape[0]
    consts = {"dl": (F32(1.0) + pD + E).astype(F32), "ebar": Ebar, "e": E,
              "sl1": (pS + E_s2).astype(F32), "sl2": (pS + E_s1).astype(F32), "mc": mc}
    acc = np.zeros((C, S), dtype=F32)
    g_pD = np.zeros(S, acc_dtype); g_pS = np.zeros(S, acc_dtype); g_mt = np.zeros(S, acc_dtype)
    g_col = np.zeros(S, acc_dtype)
    g_E = np.zeros(S, acc_dtype); g_Ebar = np.zeros(S, acc_dtype); g_Es1 = np.zeros(S, acc_dtype)
    g_Es2 = np.zeros(S, acc_dtype)
    roots = np.asarray(wl["root_row_ids"], dtype=np.int64)
    rp = Pi[roots]
    acc[roots] = -_safe_exp2_ratio(rp, lse_rows(rp)[:, None])
    leaf_state_all = np.asarray(wl["leaf_state_index"], dtype=np.int64)
    solver = so.get("self_loop_solver", "neumann")
    if relres is not None:
        row_item = np.asarray(wl["item_idx"], dtype=np.int64)
        n_fam = int(row_item.max()) + 1 if row_item.size else 0
        relres["relres"] = np.zeros(n_fam, F32)
        relres["vk_mag"] = np.zeros(n_fam, F32)
    thr = float(so.get("adjoint_pruning_threshold", 1e-6))
    prune = bool(so.get("use_adjoint_pruning", True))
    for meta in reversed(wl["wave_metas"]):
        ws, W = int(meta["start"]), int(meta["W"])
        rhs = acc[ws:ws + W]
        act = active_mask(rhs, thr, prune)
        has_splits = "sl" in meta
        dts_r = dts_forward(Pi, Pibar, meta, pD, pS, tree, active=act) if has_splits else None
        last = np.zeros(W, F32) if relres is not None else None
        v_k, aw0, aw1, aw2, aw345, aw3, aw4 = wave_backward(
            Pi, Pibar, row_max, ws, W, dts_r, rhs, consts, col_logp, tree,
            neumann_terms=int(so["neumann_terms"]),
            leaf_state=None if has_splits else leaf_state_all[ws:ws + W],
            leaf_logp=pS, active=act, grad_col=g_col, use_col_weights=use_col_weights,
            self_loop_solver=solver, last_out=last)
        if relres is not None:
            items = row_item[ws:ws + W]
            vn = np.where(act, np.sqrt((np.nan_to_num(v_k).astype(np.float64) ** 2).sum(axis=-1)), 0.0)
            np.maximum.at(relres["vk_mag"], items, vn.astype(F32))
            if str(solver).strip().lower() == "neumann" and int(so["neumann_terms"]) > 0:
                np.maximum.at(relres["relres"], items, last)
        if cache is not None:
            cache.append(dict(ws=ws, W=W, v=np.where(act[:, None], v_k, F32(0.0)).astype(F32), dts_r=dts_r,
                              active=act, has_splits=has_splits, meta=meta))
        g_pD += aw0.sum(0, dtype=F32); g_pS += aw345.sum(0, dtype=F32)
        g_E += (aw0 + aw2).sum(0, dtype=F32); g_Ebar += aw1.sum(0, dtype=F32)
        g_Es1 += aw4.sum(0, dtype=F32); g_Es2 += aw3.sum(0, dtype=F32)
        g_mt += aw2.sum(0, dtype=F32)
        if has_splits:
            ud, A, side = dts_cross_backward(Pi, Pibar, v_k, ws, meta, pD, pS, tree, acc,
                                             active=act, grad_log_pD=g_pD, grad_log_pS=g_pS,
                                             grad_mt=g_mt, mt=mc, row_max_all=row_max,
                                             side_threshold=float(so.get("pibar_side_threshold", 0.0)))
            pibar_vjp_tree(Pi, col_logp, ud, A, side, meta, tree, acc, active=act,
                           row_max_all=row_max, grad_col=g_col, use_col_weights=use_col_weights)
    out = {"pD": g_pD, "pS": g_pS, "mt": g_mt, "E": g_E, "Ebar": g_Ebar, "E_s1": g_Es1, "E_s2": g_Es2,
           "col": g_col}
    return {k: v.astype(F32) for k, v in out.items()}


def e_adjoint_and_theta_vjp(static, theta, col_weights, saved, tree: Tree, g_E, g_Ebar, g_Es1,
                            g_Es2, g_pD, g_pS, g_mt, g_col, *, n_fam, out: dict | None = None):
    """``kbench/api/_implicit_grad.py:373-475``: solve ``(I - J_E^T) wE = q_E`` by BiCGSTAB with
    E-step VJPs as the matvec, then the theta/column-weight VJP."""
    so = static["solver_options"]
    S = tree.S
    E = _f(saved["E"]).reshape(-1)
    pS = _f(saved["log_pS"]).reshape(-1); pD = _f(saved["log_pD"]).reshape(-1)
    pL = _f(saved["log_pL"]).reshape(-1); mc = _f(saved["max_coupling"]).reshape(-1)
    col_logp = _f(saved["col_log_probs"]).reshape(-1)
    ucw = not col_weights_are_uniform(col_weights)
    E_new, Es1, Es2, Ebar, _ = e_step_forward(E, pS, pD, pL, mc, col_logp, tree, ucw)
    zeros = np.zeros(S, F32)

    def vjp_E(g_new, g1, g2, gb):
        return e_step_vjp(E, E_new, Es1, Es2, Ebar, pS, pD, pL, col_logp, tree, g_new, g1, g2, gb,
                          use_col_weights=ucw)

    ge_aux = vjp_E(zeros, g_Es1, g_Es2, g_Ebar)[0]
    norm = F32(1.0) - F32(np.exp2(E).mean(dtype=F32))
    tiny = np.finfo(np.float32).tiny
    # d/dE of sum over items of log2(clamp(norm)); E has one item row shared by n_fam roots
    mult = F32(1.0) if n_fam == 1 else F32(n_fam)
    d_direct = np.where(norm > tiny, -np.exp2(E) / (F32(S) * max(norm, tiny)), F32(0.0))
    aux = (ge_aux + mult * d_direct).astype(F32)
    q = (g_E + aux).astype(F32)

    def AG(w):
        return (w - vjp_E(w, zeros, zeros, zeros)[0]).astype(F32)

    wE = bicgstab(AG, q, max_iter=so.get("bicgstab_max_iter", 500),
                  tol=so.get("bicgstab_tol", 1e-7),
                  breakdown_tol=so.get("bicgstab_breakdown_tol", 1e-30))
    if out is not None:
        out["wE"] = wE
    # theta VJP: param_loss + E-step at E_star with cotangents (wE on E_new, g_Ebar on Ebar)
    _, q_pS, q_pD, q_pL, q_mt, q_col = vjp_E(wE, zeros, zeros, g_Ebar)
    grad_theta, grad_col = extract_parameters_vjp(
        theta, col_weights if col_weights is not None else np.zeros(S, F32), tree,
        g_pS + q_pS, g_pD + q_pD, q_pL, g_mt + q_mt, g_col + q_col, uniform_fast=True)
    return grad_theta, grad_col
