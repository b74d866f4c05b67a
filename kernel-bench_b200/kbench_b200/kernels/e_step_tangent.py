"""E-step tangent wrappers (reference: ``kbench/core/kernels/e_step_tangent.py``).

Same names, arguments and results as the reference's; the work runs in the sm_100a kernels of
``csrc/kb_tangent.cu``.  ``e_tangent_fixed_point`` iterates on the device (one persistent CTA)
instead of synchronising with the host after every application.
"""

from __future__ import annotations

import torch

from .. import _lib, tree
from ._common import f32, require_cuda_f32, rows_of


def _launch_e_step_tangent_2d(E, dE, log_pS_mat, log_pD_mat, log_pL_mat, max_coupling_mat, col_log_probs,
                              dlog_pS_mat, dlog_pD_mat, dlog_pL_mat, dmax_coupling_mat, node_parent, node_child1,
                              node_child2, max_ancestor_depth, *, out=None, max_diff_out=None,
                              use_col_weights=True):
    """Reference ``e_step_tangent.py:153-171``: one linearised E application per item row;
    returns ``(dE_new, dE_s1, dE_s2, dEbar)``."""
    require_cuda_f32("_launch_e_step_tangent_2d", E, dE)
    G, S = int(E.shape[0]), int(E.shape[1])
    E, dE = f32(E), f32(dE)
    dE_new, dE_s1, dE_s2, dEbar = (torch.empty_like(E) for _ in range(4)) if out is None else out
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    pS, pD, pL, mc = (rows_of(t, G, S) for t in (log_pS_mat, log_pD_mat, log_pL_mat, max_coupling_mat))
    dpS, dpD, dpL, dmc = (rows_of(t, G, S) for t in (dlog_pS_mat, dlog_pD_mat, dlog_pL_mat, dmax_coupling_mat))
    _lib.call("kb_e_tangent_step", E.data_ptr(), dE.data_ptr(), dpS.data_ptr(), dpD.data_ptr(), dpL.data_ptr(),
              dmc.data_ptr(), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), mc.data_ptr(),
              f32(col_log_probs.reshape(-1)).data_ptr(), int(bool(use_col_weights)), tt.child1.data_ptr(),
              tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K, G, S, 1, dE_new.data_ptr(), dE_s1.data_ptr(),
              dE_s2.data_ptr(), dEbar.data_ptr(), _lib.ptr(max_diff_out), _lib.stream_handle(E.device))
    return dE_new, dE_s1, dE_s2, dEbar


def e_tangent_fixed_point(E_star, dlog_pS, dlog_pD, dlog_pL, dmax_coupling, log_pS, log_pD, log_pL, max_coupling,
                          col_log_probs, node_parent, node_child1, node_child2, max_ancestor_depth, *,
                          max_iter=2000, tol=1e-9, use_col_weights=True, dE0=None):
    """Reference ``e_step_tangent.py:174-208``: solve ``(I - J_E^EE) dE* = J_E^Ep dp`` at the frozen
    ``E*`` by Richardson iteration (stop when ``max|dE_new - dE| <= tol * max(1, max|dE_new|)``);
    returns ``(dE*, dE_s1, dE_s2, dEbar)``."""
    require_cuda_f32("e_tangent_fixed_point", E_star)
    E = f32(E_star)
    G, S = int(E.shape[0]), int(E.shape[1])
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    pS, pD, pL, mc = (rows_of(t, G, S) for t in (log_pS, log_pD, log_pL, max_coupling))
    dpS, dpD, dpL, dmc = (rows_of(t, G, S) for t in (dlog_pS, dlog_pD, dlog_pL, dmax_coupling))
    dE, scratch, dE_s1, dE_s2, dEbar = (torch.empty_like(E) for _ in range(5))
    _lib.call("kb_e_tangent_fixed_point", E.data_ptr(), dpS.data_ptr(), dpD.data_ptr(), dpL.data_ptr(),
              dmc.data_ptr(), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), mc.data_ptr(),
              f32(col_log_probs.reshape(-1)).data_ptr(), int(bool(use_col_weights)), tt.child1.data_ptr(),
              tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K, G, S, 1, int(max_iter), float(tol),
              _lib.ptr(None if dE0 is None else rows_of(dE0, G, S)), dE.data_ptr(), scratch.data_ptr(),
              dE_s1.data_ptr(), dE_s2.data_ptr(), dEbar.data_ptr(), None, _lib.stream_handle(E.device))
    return dE, dE_s1, dE_s2, dEbar
