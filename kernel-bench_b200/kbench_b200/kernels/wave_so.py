"""Second-order contraction of the wave-step adjoint (reference: ``kbench/core/kernels/wave_so.py``)."""

from __future__ import annotations

import torch

from .. import _lib, tree
from ._common import f32, i32, i64, require_cuda_f32
from .wave_step import _const_row_stride


def wave_backward_so(Pi_star, dPi, Pibar_star, dPibar, v, ws, W, S, pibar_row_max, mc, DL, dDL, Ebar, dEbar, E, dE,
                     SL1, dSL1, SL2, dSL2, col_log_probs, node_child1, node_child2, node_parent, max_ancestor_depth,
                     dts_r=None, d_dts=None, *, leaf_state_idx, leaf_logp, dleaf_logp, item_idx, has_leaf_term=True,
                     use_col_weights=False, d_rhs=None):
    """Reference ``wave_so.py:213-250``: at the fixed adjoint ``v`` [W,S], the tangent of the wave's
    self-loop J^T v and of its parameter buckets.  Returns (d_Av [W,S], d_aw0, d_aw1, d_aw2, d_aw345,
    d_aw3, d_aw4); with ``d_rhs`` [C,S] the wave's rows of it are folded into ``d_Av`` (the seed of
    the reused solve)."""
    require_cuda_f32("wave_backward_so", Pi_star, dPi, Pibar_star, dPibar, v, dts_r, d_dts, d_rhs)
    ws, W, S = int(ws), int(W), int(S)
    if (dts_r is None) != (d_dts is None):
        raise ValueError("wave_backward_so: dts_r and d_dts must be given together")
    dev = Pi_star.device
    d_out = torch.empty((W, S), device=dev, dtype=torch.float32)
    d_aw = torch.empty((6, W, S), device=dev, dtype=torch.float32)
    if W == 0:
        return (d_out, *d_aw.unbind(0))
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    consts = [f32(t) for t in (mc, DL, dDL, Ebar, dEbar, E, dE, SL1, dSL1, SL2, dSL2)]
    crs = _const_row_stride(consts[1])
    _lib.call("kb_wave_backward_so", f32(Pi_star).data_ptr(), f32(dPi).data_ptr(), f32(Pibar_star).data_ptr(),
              f32(dPibar).data_ptr(), f32(v).data_ptr(), ws, W, f32(pibar_row_max).data_ptr(),
              *[c.data_ptr() for c in consts], crs, f32(col_log_probs).data_ptr(), int(bool(use_col_weights)),
              tt.parent.data_ptr(), tt.child1.data_ptr(), tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K,
              _lib.ptr(tt.lv_ptr), tt.n_levels, _lib.ptr(tt.lv_par), _lib.ptr(tt.lv_c1), _lib.ptr(tt.lv_c2),
              i32(leaf_state_idx).data_ptr() if has_leaf_term else None, f32(leaf_logp).data_ptr(),
              f32(dleaf_logp).data_ptr(), i64(item_idx).data_ptr(), _lib.ptr(f32(dts_r)), _lib.ptr(f32(d_dts)),
              _lib.ptr(d_rhs), d_out.data_ptr(), d_aw.data_ptr(), S, _lib.stream_handle(dev))
    return (d_out, *d_aw.unbind(0))
