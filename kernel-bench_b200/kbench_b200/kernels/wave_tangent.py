"""Wave-step tangent wrappers (reference: ``kbench/core/kernels/wave_tangent.py``)."""

from __future__ import annotations

from .. import _lib, tree
from ._common import f32, i32, i64, require_cuda_f32
from .wave_step import _const_row_stride


def _launch(name, Pi_in, dPi_in, dPi_out, ws, W, S, n_iters, consts, col_log_probs, node_child1, node_child2,
            node_parent, max_ancestor_depth, DTS_reduced, dDTS, leaf_state_idx, leaf_logp, dleaf_logp, item_idx,
            dPibar_out, has_leaf_term, input_ws, use_col_weights):
    require_cuda_f32(name, Pi_in, dPi_in, dPi_out, dPibar_out, DTS_reduced, dDTS)
    ws, W, S = int(ws), int(W), int(S)
    if W == 0:
        return
    if (DTS_reduced is None) != (dDTS is None):
        raise ValueError(f"{name}: DTS_reduced and dDTS must be given together")
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    mc, dmc, dl, ddl, eb, deb, e, de, s1, ds1, s2, ds2 = (f32(t) for t in consts)
    crs = _const_row_stride(dl)
    out_rows = dPi_out.data_ptr() + ws * int(dPi_out.stride(0)) * 4
    pi_ws = ws if input_ws is None else int(input_ws)
    _lib.call("kb_wave_tangent", f32(Pi_in).data_ptr(), f32(dPi_in).data_ptr(), out_rows, _lib.ptr(dPibar_out),
              ws, pi_ws, W, S, int(n_iters), mc.data_ptr(), dmc.data_ptr(), dl.data_ptr(), ddl.data_ptr(),
              eb.data_ptr(), deb.data_ptr(), e.data_ptr(), de.data_ptr(), s1.data_ptr(), ds1.data_ptr(),
              s2.data_ptr(), ds2.data_ptr(), crs, f32(col_log_probs).data_ptr(), int(bool(use_col_weights)),
              tt.child1.data_ptr(), tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K,
              i32(leaf_state_idx).data_ptr() if has_leaf_term else None, f32(leaf_logp).data_ptr(),
              f32(dleaf_logp).data_ptr(), i64(item_idx).data_ptr(), _lib.ptr(f32(DTS_reduced)),
              _lib.ptr(f32(dDTS)), _lib.stream_handle(Pi_in.device))


def compute_wave_step_tangent_selfloop(Pi_in, dPi_io, ws, W, S, n_iters, max_coupling_mat, dMC, DL, dDL, Ebar, dEbar,
                                       E, dE, SL1, dSL1, SL2, dSL2, col_log_probs, node_child1, node_child2,
                                       node_parent, max_ancestor_depth, DTS_reduced=None, dDTS=None, *,
                                       leaf_state_idx, leaf_logp, dleaf_logp, item_idx, dPibar_out=None,
                                       has_leaf_term=True, use_col_weights=True):
    """Reference ``wave_tangent.py:339-389``: ``n_iters`` in-place Jacobi steps of the linearised
    wave step on ``dPi_io[ws:ws+W]`` in one launch; ``dPibar_out[ws:ws+W]`` from the last step."""
    _launch("compute_wave_step_tangent_selfloop", Pi_in, dPi_io, dPi_io, ws, W, S, max(int(n_iters), 1),
            (max_coupling_mat, dMC, DL, dDL, Ebar, dEbar, E, dE, SL1, dSL1, SL2, dSL2), col_log_probs, node_child1,
            node_child2, node_parent, max_ancestor_depth, DTS_reduced, dDTS, leaf_state_idx, leaf_logp, dleaf_logp,
            item_idx, dPibar_out, has_leaf_term, None, use_col_weights)


def compute_wave_step_tangent(Pi_in, dPi_in, dPi_out, ws, W, S, max_coupling_mat, dMC, DL, dDL, Ebar, dEbar, E, dE,
                              SL1, dSL1, SL2, dSL2, col_log_probs, node_child1, node_child2, node_parent,
                              max_ancestor_depth, DTS_reduced=None, dDTS=None, *, leaf_state_idx, leaf_logp,
                              dleaf_logp, item_idx, dPibar_out=None, has_leaf_term=True, input_ws=None,
                              use_col_weights=True):
    """Reference ``wave_tangent.py:392-431``: one tangent application; writes ``dPi_out[ws:ws+W]``
    (reading ``Pi_in`` / ``dPi_in`` rows at ``input_ws`` or ``ws``) and optionally ``dPibar_out``."""
    _launch("compute_wave_step_tangent", Pi_in, dPi_in, dPi_out, ws, W, S, 1,
            (max_coupling_mat, dMC, DL, dDL, Ebar, dEbar, E, dE, SL1, dSL1, SL2, dSL2), col_log_probs, node_child1,
            node_child2, node_parent, max_ancestor_depth, DTS_reduced, dDTS, leaf_state_idx, leaf_logp, dleaf_logp,
            item_idx, dPibar_out, has_leaf_term, input_ws, use_col_weights)
