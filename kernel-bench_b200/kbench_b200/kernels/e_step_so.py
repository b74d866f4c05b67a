"""Second-order contraction of the E-step backward (reference: ``kbench/core/kernels/e_step_so.py``)."""

from __future__ import annotations

import torch

from .. import _lib, tree
from ._common import f32, require_cuda_f32, rows_of


def e_step_backward_so(E, E_new, E_s1, E_s2, Ebar, log_pS, log_pD, log_pL, col_log_probs, node_parent, node_child1,
                       node_child2, max_ancestor_depth, g_new, g_s1, g_s2, g_ebar, dE, dE_new, dE_s1, dE_s2, dEbar,
                       dlog_pS, dlog_pD, dlog_pL, dcol, *, use_col_weights=False):
    """Reference ``e_step_so.py:188-220``: (d/dx of the E-step backward)(x; g) . dx at fixed
    cotangents.  Returns (d_grad_E, d_grad_pS, d_grad_pD, d_grad_pL, d_grad_mc, d_grad_col);
    ``g_s1`` / ``g_s2`` enter the backward linearly and are accepted for interface symmetry."""
    require_cuda_f32("e_step_backward_so", E, E_new, E_s1, E_s2, Ebar, g_new, g_ebar, dE, dE_new)
    G, S = int(E.shape[0]), int(E.shape[1])
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    rows = [rows_of(t, G, S) for t in (E, E_new, E_s1, E_s2, Ebar, log_pS, log_pD, log_pL, g_new, g_ebar, dE, dE_new,
                                       dE_s1, dE_s2, dEbar, dlog_pS, dlog_pD, dlog_pL)]
    outs = [torch.empty((G, S), device=E.device, dtype=torch.float32) for _ in range(5)]
    d_grad_col = torch.empty_like(f32(col_log_probs.reshape(-1)))
    _lib.call("kb_e_step_backward_so", *[t.data_ptr() for t in rows[:8]], f32(col_log_probs.reshape(-1)).data_ptr(),
              tt.parent.data_ptr(), tt.child1.data_ptr(), tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K,
              _lib.ptr(tt.lv_ptr), tt.n_levels, _lib.ptr(tt.lv_par), _lib.ptr(tt.lv_c1), _lib.ptr(tt.lv_c2),
              *[t.data_ptr() for t in rows[8:]], _lib.ptr(None if dcol is None else f32(dcol.reshape(-1))),
              *[t.data_ptr() for t in outs], d_grad_col.data_ptr(), S, G, int(bool(use_col_weights)),
              _lib.stream_handle(E.device))
    return (*outs, d_grad_col.reshape(col_log_probs.shape))
