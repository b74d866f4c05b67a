"""Split reduction wrapper (reference: ``kbench/core/kernels/dts_fused.py``)."""

from __future__ import annotations

import torch

from .. import _lib
from ._common import f32, i32, i64, require_cuda_f32, state_rows, u8


def compute_dts_forward(Pi, Pibar, lefts, rights, node_child1, node_child2, W, reduce_idx, log_pD_vec,
                        log_pS_vec, item_idx, *, log_split_probs=None, n_eq1=None, eq1_reduce_idx=None,
                        ge2_ptr=None, ge2_parent_ids=None, ge2_max_fanout=None, active_parent_rows=None,
                        item_offset=0):
    """Reference ``dts_fused.py:171-231``: returns a new [W,S] tensor, -inf on rows of inactive
    (or split-less) parents. ``ge2_max_fanout`` is accepted for signature compatibility; the
    sm_100a kernel walks each parent's splits directly and needs no tile count."""
    require_cuda_f32("compute_dts_forward", Pi, Pibar)
    N = int(lefts.shape[0])
    S = int(Pi.shape[1])
    W = int(W)
    out = torch.full((W, S), float("-inf"), device=Pi.device, dtype=Pi.dtype)
    if N == 0 or W == 0:
        return out
    if log_split_probs is None:
        lsp = torch.zeros((N,), device=Pi.device, dtype=Pi.dtype)
    else:
        lsp = f32(log_split_probs.reshape(N))
    if n_eq1 is None:
        n_eq1 = N
        eq1_reduce_idx = reduce_idx
        ge2_parent_ids = None
        ge2_ptr = None
    n_eq1 = int(n_eq1)
    n_ge2 = 0 if ge2_parent_ids is None else int(ge2_parent_ids.numel())
    pD, prs = state_rows(log_pD_vec, S)
    pS, prs2 = state_rows(log_pS_vec, S)
    if prs != prs2:
        raise ValueError("log_pD/log_pS must use the same layout")
    _lib.call("kb_dts_forward", f32(Pi).data_ptr(), f32(Pibar).data_ptr(), i64(lefts).data_ptr(),
              i64(rights).data_ptr(), i32(node_child1).data_ptr(), i32(node_child2).data_ptr(),
              pD.data_ptr(), pS.data_ptr(), prs, i64(item_idx).data_ptr(), int(item_offset), lsp.data_ptr(),
              _lib.ptr(i64(eq1_reduce_idx)) if n_eq1 else None, n_eq1,
              _lib.ptr(i64(ge2_ptr)) if n_ge2 else None, _lib.ptr(i64(ge2_parent_ids)) if n_ge2 else None,
              n_ge2, _lib.ptr(u8(active_parent_rows)), out.data_ptr(), None, S, _lib.stream_handle(Pi.device))
    return out
