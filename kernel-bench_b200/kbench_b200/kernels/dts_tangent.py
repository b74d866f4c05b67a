"""Split-reduction tangent wrapper (reference: ``kbench/core/kernels/dts_tangent.py``)."""

from __future__ import annotations

import torch

from .. import _lib
from ._common import f32, i32, i64, require_cuda_f32, state_rows


def parent_csr(reduce_idx, W):
    """(order, ptr): the splits of each of the W parent rows, in split order, as a CSR over
    ``reduce_idx`` -- the fixed summation order of :func:`compute_dts_tangent`.  Depends only on the
    wave layout, so callers that run many tangents can build it once and pass it as ``csr``."""
    N = int(reduce_idx.numel())
    red = i64(reduce_idx.reshape(N))
    order = torch.sort(red, stable=True).indices.contiguous()
    counts = torch.bincount(red, minlength=int(W))
    ptr = torch.zeros((int(W) + 1,), device=red.device, dtype=torch.int64)
    torch.cumsum(counts, 0, out=ptr[1:])
    return order, ptr


def compute_dts_tangent(Pi, Pibar, dPi, dPibar, lefts, rights, node_child1, node_child2, W, reduce_idx,
                        log_pD_vec, log_pS_vec, dlog_pD_vec, dlog_pS_vec, dts_r, item_idx, *, log_split_probs=None,
                        n_eq1=None, eq1_reduce_idx=None, ge2_ptr=None, ge2_parent_ids=None, ge2_max_fanout=None,
                        item_offset=0, csr=None):
    """Reference ``dts_tangent.py:99-122``: returns a new ``d_dts`` [W,S].  Each parent row sums its
    splits in a fixed order (the eq1 / ge2 layout arguments are accepted for signature
    compatibility; the full ``reduce_idx`` map is used, as the reference's kernel does).  ``csr``:
    :func:`parent_csr` of this wave, built once by the caller (else here)."""
    require_cuda_f32("compute_dts_tangent", Pi, Pibar, dPi, dPibar, dts_r)
    N = int(lefts.shape[0])
    S = int(Pi.shape[1])
    W = int(W)
    out = torch.zeros((W, S), device=Pi.device, dtype=Pi.dtype)
    if N == 0 or W == 0:
        return out
    order, ptr = parent_csr(reduce_idx, W) if csr is None else csr
    lsp = None if log_split_probs is None else f32(log_split_probs.reshape(N))
    pD, prs = state_rows(log_pD_vec, S)
    pS, _ = state_rows(log_pS_vec, S)
    dpD, _ = state_rows(dlog_pD_vec, S)
    dpS, _ = state_rows(dlog_pS_vec, S)
    _lib.call("kb_dts_tangent", f32(Pi).data_ptr(), f32(Pibar).data_ptr(), f32(dPi).data_ptr(),
              f32(dPibar).data_ptr(), i64(lefts).data_ptr(), i64(rights).data_ptr(), _lib.ptr(lsp),
              order.data_ptr(), ptr.data_ptr(), W, i32(node_child1).data_ptr(), i32(node_child2).data_ptr(),
              pD.data_ptr(), pS.data_ptr(), dpD.data_ptr(), dpS.data_ptr(), prs, i64(item_idx).data_ptr(),
              int(item_offset), f32(dts_r).data_ptr(), out.data_ptr(), S, _lib.stream_handle(Pi.device))
    return out
