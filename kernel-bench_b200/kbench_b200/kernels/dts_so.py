"""Second-order contraction of the split backward (reference: ``kbench/core/kernels/dts_so.py``)."""

from __future__ import annotations

import torch

from .. import _lib, tree
from ._common import f32, i64, require_cuda_f32, state_rows


def _inplace(name, t):
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise RuntimeError(f"dts_backward_so: {name} must be a contiguous fp32 tensor (accumulated in place)")
    return t


def dts_backward_so(Pi, dPi, Pibar, dPibar, v, ws, meta, S, log_pD_param, log_pS_param, dlog_pD_param, dlog_pS_param,
                    mc_item, dmc_item, col_log_probs, node_child1, node_child2, node_parent, max_ancestor_depth,
                    pibar_row_max, item_idx, d_rhs, d_grad_pD, d_grad_pS, d_grad_mt, d_grad_col, *,
                    compact_level_ptr=None, compact_level_parents=None, compact_level_child1=None,
                    compact_level_child2=None, use_col_weights=False):
    """Reference ``dts_so.py:233-303``: the second-order contraction of the wave's split backward
    and Pibar VJP trees at the fixed adjoint ``v`` [W,S]; accumulates into ``d_rhs`` [C,S] and the
    ``d_grad_*`` buffers in place."""
    require_cuda_f32("dts_backward_so", Pi, dPi, Pibar, dPibar, v, d_rhs, d_grad_pD, d_grad_pS, d_grad_mt,
                     d_grad_col)
    sl, sr = meta["sl"], meta["sr"]
    N = int(sl.numel())
    if N == 0:
        return
    S = int(S)
    for name, t in (("d_rhs", d_rhs), ("d_grad_pD", d_grad_pD), ("d_grad_pS", d_grad_pS),
                    ("d_grad_mt", d_grad_mt), ("d_grad_col", d_grad_col)):
        _inplace(name, t)
    lsp = meta.get("log_split_probs")
    lsp = None if lsp is None else f32(lsp.reshape(N))
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth,
                     compact_level_ptr=compact_level_ptr, compact_level_parents=compact_level_parents,
                     compact_level_child1=compact_level_child1, compact_level_child2=compact_level_child2)
    pD, prs = state_rows(log_pD_param, S)
    pS, _ = state_rows(log_pS_param, S)
    dpD, _ = state_rows(dlog_pD_param, S)
    dpS, _ = state_rows(dlog_pS_param, S)
    mt, mrs = state_rows(mc_item, S)
    dmt, _ = state_rows(dmc_item, S)
    dev = Pi.device
    ud = torch.empty((2 * N, S), device=dev, dtype=torch.float32)
    dud = torch.empty((2 * N, S), device=dev, dtype=torch.float32)
    _lib.call("kb_dts_backward_so", f32(Pi).data_ptr(), f32(dPi).data_ptr(), f32(Pibar).data_ptr(),
              f32(dPibar).data_ptr(), f32(v).data_ptr(), int(ws), i64(sl).data_ptr(), i64(sr).data_ptr(),
              i64(meta["reduce_idx"]).data_ptr(), _lib.ptr(lsp), N, int(meta["start"]), i64(item_idx).data_ptr(),
              pD.data_ptr(), pS.data_ptr(), dpD.data_ptr(), dpS.data_ptr(), prs, mt.data_ptr(), dmt.data_ptr(), mrs,
              f32(pibar_row_max).data_ptr(), f32(col_log_probs).data_ptr(), int(bool(use_col_weights)),
              tt.child1.data_ptr(), tt.child2.data_ptr(), _lib.ptr(tt.lv_ptr), tt.n_levels, _lib.ptr(tt.lv_par),
              _lib.ptr(tt.lv_c1), _lib.ptr(tt.lv_c2), ud.data_ptr(), dud.data_ptr(), d_rhs.data_ptr(),
              d_grad_pD.data_ptr(), d_grad_pS.data_ptr(), d_grad_mt.data_ptr(), d_grad_col.data_ptr(), S,
              _lib.stream_handle(dev))
