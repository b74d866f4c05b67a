"""Forward wave wrappers (reference: ``kbench/core/kernels/wave_step.py``)."""

from __future__ import annotations

from .. import _lib, tree
from ._common import f32, i32, i64, require_cuda_f32


def _const_row_stride(const_tensor) -> int:
    """Reference ``wave_step.py:19-22``: a one-row constant is shared by every item."""
    return 0 if int(const_tensor.shape[0]) == 1 else int(const_tensor.stride(0))


def compute_leaf_initial_wave_step(Pi_out, ws, W, S, max_coupling_mat, DL_const, Ebar, E, SL1_const, SL2_const,
                                   col_log_probs, node_child1, node_child2, node_subtree_start,
                                   node_subtree_end, leaf_state_idx, leaf_logp, item_idx, use_col_weights=True):
    """Reference ``wave_step.py:1078-1126``: seeds rows [ws, ws+W) of ``Pi_out`` in place."""
    require_cuda_f32("compute_leaf_initial_wave_step", Pi_out)
    ws, W, S = int(ws), int(W), int(S)
    if W == 0:
        return
    out_rows = Pi_out.data_ptr() + ws * int(Pi_out.stride(0)) * 4
    _lib.call("kb_leaf_initial", out_rows, f32(max_coupling_mat).data_ptr(), f32(DL_const).data_ptr(),
              f32(Ebar).data_ptr(), f32(E).data_ptr(), f32(SL1_const).data_ptr(), f32(SL2_const).data_ptr(),
              _const_row_stride(DL_const), f32(col_log_probs).data_ptr(), int(bool(use_col_weights)),
              i32(node_child1).data_ptr(), i32(node_child2).data_ptr(), i32(node_subtree_start).data_ptr(),
              i32(node_subtree_end).data_ptr(), i32(leaf_state_idx).data_ptr(), f32(leaf_logp).data_ptr(),
              i64(item_idx).data_ptr(), ws, W, S, _lib.stream_handle(Pi_out.device))


def compute_wave_step(Pi_in, Pi_out, Pibar, ws, W, S, max_coupling_mat, DL_const, Ebar, E, SL1_const, SL2_const,
                      col_log_probs, node_child1, node_child2, node_parent, max_ancestor_depth, DTS_reduced=None,
                      *, leaf_state_idx, leaf_logp, item_idx, pibar_row_max, store_final_pibar=False,
                      has_leaf_term=True, input_ws=None, use_col_weights=True, pi_residual_out=None):
    """Reference ``wave_step.py:1128-1268``: one Jacobi sweep of rows [ws, ws+W).

    Reads ``Pi_in`` rows [input_ws or ws, +W), writes ``Pi_out`` rows [ws, ws+W); on the final
    iteration (``store_final_pibar``) also writes ``Pibar`` rows and ``pibar_row_max``.  The
    argument aliasing used by ``kbench/core/inference/forward.py`` (Pi_out or Pi_in being the same
    buffer as Pibar) is safe: each row is staged in shared memory before any of its outputs is
    written."""
    require_cuda_f32("compute_wave_step", Pi_in, Pi_out, Pibar)
    ws, W, S = int(ws), int(W), int(S)
    if W == 0:
        return
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    pi_ws = ws if input_ws is None else int(input_ws)
    out_rows = Pi_out.data_ptr() + ws * int(Pi_out.stride(0)) * 4
    _lib.call("kb_wave_step", Pi_in.data_ptr(), pi_ws, out_rows, Pibar.data_ptr(), pibar_row_max.data_ptr(),
              _lib.ptr(pi_residual_out), _lib.ptr(None if DTS_reduced is None else f32(DTS_reduced)),
              f32(max_coupling_mat).data_ptr(), f32(DL_const).data_ptr(), f32(Ebar).data_ptr(),
              f32(E).data_ptr(), f32(SL1_const).data_ptr(), f32(SL2_const).data_ptr(),
              _const_row_stride(DL_const), f32(col_log_probs).data_ptr(), int(bool(use_col_weights)),
              tt.child1.data_ptr(), tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K,
              i32(leaf_state_idx).data_ptr(), f32(leaf_logp).data_ptr(), i64(item_idx).data_ptr(),
              int(bool(has_leaf_term)), int(bool(store_final_pibar)), ws, W, S, _lib.stream_handle(Pi_in.device))
