"""Backward (implicit adjoint) wrappers (reference: ``kbench/core/kernels/wave_backward.py``)."""

from __future__ import annotations

import torch

from .. import _lib, tree
from ._common import f32, i32, i64, require_cuda_f32, u8

_SUPPORTED = (torch.float32,)


def active_mask_from_rhs_absmax_fused(rhs, threshold, *, use_pruning=True):
    """Reference ``wave_backward.py:247-280``: ``max|rhs[w]| >= threshold`` (``>`` when pruning is
    off)."""
    if rhs.ndim != 2:
        raise ValueError("rhs must be a 2D tensor")
    if rhs.device.type != "cuda":
        raise ValueError("active_mask_from_rhs_absmax_fused requires a CUDA tensor")
    if rhs.dtype not in _SUPPORTED:
        raise ValueError("active_mask_from_rhs_absmax_fused supports fp32 tensors")
    W, S = int(rhs.shape[0]), int(rhs.shape[1])
    mask = torch.empty((W,), device=rhs.device, dtype=torch.bool)
    if W == 0:
        return mask
    if rhs.stride(1) != 1:
        rhs = rhs.contiguous()
    _lib.call("kb_active_mask", rhs.data_ptr(), int(rhs.stride(0)), W, S, float(threshold),
              int(not use_pruning), mask.data_ptr(), _lib.stream_handle(rhs.device))
    return mask


def _const_mode(const_tensor, item_idx, item_indexed):
    """Reference ``wave_backward.py:103-120``."""
    if item_indexed:
        if item_idx is None:
            raise ValueError("item-indexed backward constants require item_idx")
        if const_tensor.ndim != 2:
            raise ValueError("item-indexed backward constants require [G, S] tensors")
        return 2
    return 1 if const_tensor.ndim == 2 else 0


def _leaf_mode(use_leaf_index, leaf_logp, item_idx, item_indexed):
    """Reference ``wave_backward.py:123-140``."""
    if not use_leaf_index:
        return 0
    if item_indexed:
        if item_idx is None:
            raise ValueError("item-indexed leaf log-probabilities require item_idx")
        if leaf_logp.ndim == 1:
            return 1
        if leaf_logp.ndim == 2:
            if int(leaf_logp.shape[1]) == 1:
                raise ValueError("item-indexed [G, 1] leaf_logp should be expanded to [G, S]")
            return 2
        raise ValueError("item-indexed leaf_logp must have shape [G] or [G, S]")
    if leaf_logp.numel() == 1:
        return 3
    return 0


def _gmres_fixed(apply_a, b, max_iter: int):
    """Solve ``A v = b`` by unrestarted GMRES with a fixed number of Arnoldi steps, the whole wave
    ``[W,S]`` being ONE vector (reference ``wave_backward.py:831-912``): the Krylov basis is built
    by classical Gram-Schmidt with one re-orthogonalisation pass, the iteration stops early when
    the new basis vector's norm falls to ``eps * max(|b|, 1)``, and ``v`` minimises the residual
    through the least-squares solve of the small Hessenberg system.  ``apply_a`` (one launch of
    the row operator) runs on the device; the dense orthogonalisation is a few matrix-vector
    products over the basis."""
    m = int(max_iter)
    if m < 1:
        return torch.zeros_like(b)
    beta = torch.linalg.vector_norm(b)
    if float(beta) == 0.0:
        return torch.zeros_like(b)
    dt, dev = b.dtype, b.device
    basis = torch.empty((m + 1, b.numel()), dtype=dt, device=dev)
    basis[0] = b.reshape(-1) / beta
    hess = torch.zeros((m + 1, m), dtype=dt, device=dev)
    g = torch.zeros((m + 1,), dtype=dt, device=dev)
    g[0] = beta
    steps = m
    stop = torch.finfo(dt).eps * torch.clamp(beta, min=1.0)
    for j in range(m):
        w = apply_a(basis[j].view(b.shape)).reshape(-1)
        q = basis[: j + 1]
        h1 = torch.mv(q, w)
        w1 = torch.addmv(w, q.t(), h1, beta=1.0, alpha=-1.0)
        h2 = torch.mv(q, w1)
        w2 = torch.addmv(w1, q.t(), h2, beta=1.0, alpha=-1.0)
        hess[: j + 1, j] = h1 + h2
        nrm = torch.linalg.vector_norm(w2)
        hess[j + 1, j] = nrm
        if bool(nrm <= stop):
            steps = j + 1
            break
        if j + 1 < m:
            basis[j + 1] = w2 / torch.clamp(nrm, min=torch.finfo(dt).tiny)
    y = torch.linalg.lstsq(hess[: steps + 1, :steps], g[: steps + 1]).solution
    return torch.mv(basis[:steps].t(), y).view(b.shape)


def wave_backward_uniform_fused(Pi_star, Pibar_star, ws, W, S, dts_r, rhs, mt_squeezed, DL_const, Ebar, E,
                                SL1_const, SL2_const, col_log_probs, node_child1, node_child2, leaf_term_wt,
                                neumann_terms=3, leaf_state_idx=None, leaf_logp=None, has_leaf_term=True,
                                active_mask=None, node_parent=None, max_ancestor_depth=None, pibar_row_max=None,
                                item_idx=None, item_indexed_consts=False, compact_level_ptr=None,
                                compact_level_parents=None, compact_level_child1=None, compact_level_child2=None,
                                grad_col_log_probs=None, use_col_weights=True, self_loop_grad_targets=None,
                                initial_v=None, self_loop_solver="neumann", return_last_increment=False):
    """Reference ``wave_backward.py:1737-1867``: per active row, the adjoint ``v`` of the self-loop
    -- ``self_loop_solver="neumann"``: the series ``v = sum_{n=0..N} (J_self^T)^n rhs``, or, given
    ``initial_v`` ([W,S]), ``v = initial_v`` followed by ``N`` fixed-point updates
    ``v <- rhs + J_self^T v`` (``:1493-1534``; inactive rows keep ``initial_v``); ``"gmres"``: ``N``
    GMRES steps on ``(I - J_self^T) v = rhs`` over the whole wave -- and the per-element parameter
    cotangents.

    Returns ``(v_k, aw0, aw1, aw2, aw345, aw3, aw4)`` (new [W,S] tensors; aw* zero and v_k
    unspecified on inactive rows in the Neumann solve, zero in the GMRES solve), plus, with
    ``return_last_increment``, the per-row ``|last Neumann term| / |v|`` ([W], zero on inactive
    rows; None for the GMRES solve, a warm-started solve or N = 0, as the reference); accumulates
    ``grad_col_log_probs`` in place.  With ``self_loop_grad_targets`` = (grad_log_pD, grad_log_pS,
    grad_E, grad_Ebar, grad_E_s1, grad_E_s2, grad_mt, param_grad_vector) (``:1615-1640``, ``:1208-1262``)
    the buckets' column sums over the wave are added into those fp32 tensors instead (pD += aw0,
    pS += aw345 -- per column with ``param_grad_vector``, else one scalar each --, E += aw0 + aw2,
    Ebar += aw1, E_s1 += aw4, E_s2 += aw3, mt += aw2) and the six buckets are returned as None."""
    require_cuda_f32("GPUREC self-loop 2D fast path", Pi_star, Pibar_star, rhs)
    solver = str(self_loop_solver).strip().lower()
    if solver not in ("neumann", "gmres"):
        raise ValueError(f"unsupported self-loop solver {self_loop_solver!r}")
    if solver == "gmres" and initial_v is not None:
        raise ValueError("GMRES self-loop solve does not support initial_v")
    targets = _grad_targets(self_loop_grad_targets, int(S), Pi_star.device)
    requested_has_leaf_term = bool(has_leaf_term)
    use_leaf_index = requested_has_leaf_term and leaf_state_idx is not None and leaf_logp is not None
    const_mode = _const_mode(DL_const, item_idx, bool(item_indexed_consts))
    if bool(item_indexed_consts) and use_leaf_index:
        if leaf_logp.ndim == 1:
            leaf_logp = leaf_logp.unsqueeze(-1).expand(-1, S).contiguous()
        elif leaf_logp.ndim == 2 and int(leaf_logp.shape[1]) == 1:
            leaf_logp = leaf_logp.expand(-1, S).contiguous()
    leaf_mode = _leaf_mode(use_leaf_index, leaf_logp, item_idx, bool(item_indexed_consts))
    if node_parent is None:
        raise ValueError("node_parent is required for the retained backward fast path")
    if max_ancestor_depth is None:
        raise ValueError("max_ancestor_depth is required for the retained backward fast path")
    if pibar_row_max is None:
        raise ValueError("pibar_row_max is required for the retained backward fast path")
    if compact_level_ptr is None or compact_level_parents is None or compact_level_child1 is None \
            or compact_level_child2 is None:
        raise ValueError("compact state levels are required for the retained 2D self-loop path")
    ws, W, S = int(ws), int(W), int(S)
    dev = Pi_star.device
    tt = tree.tables(node_parent, node_child1, node_child2, int(max_ancestor_depth),
                     compact_level_ptr=compact_level_ptr, compact_level_parents=compact_level_parents,
                     compact_level_child1=compact_level_child1, compact_level_child2=compact_level_child2)
    shape = (W, S)
    v_k, aw0, aw1, aw2, aw345, aw3, aw4 = (torch.empty(shape, device=dev, dtype=torch.float32) for _ in range(7))
    if initial_v is not None:
        if tuple(initial_v.shape) != shape:
            raise ValueError(f"initial_v shape {tuple(initial_v.shape)} does not match wave scratch shape {shape}")
        initial_v = initial_v.to(device=dev, dtype=torch.float32).contiguous()
    want_rel = (bool(return_last_increment) and solver == "neumann" and initial_v is None
                and int(neumann_terms) > 0)
    last_rel = torch.empty((W,), device=dev, dtype=torch.float32) if want_rel else None
    out = (v_k, aw0, aw1, aw2, aw345, aw3, aw4) if targets is None else (v_k, None, None, None, None, None, None)
    if W == 0:
        if initial_v is not None:
            v_k.copy_(initial_v)
        return (*out, last_rel) if return_last_increment else out
    has_materialized = leaf_term_wt is not None
    leaf_term = None
    if requested_has_leaf_term and not use_leaf_index and has_materialized:
        leaf_term = f32(leaf_term_wt)
    st = _lib.stream_handle(dev)
    mask_u8 = u8(active_mask)
    head = (f32(Pi_star).data_ptr(), f32(Pibar_star).data_ptr(), f32(pibar_row_max).data_ptr(),
            _lib.ptr(None if dts_r is None else f32(dts_r)))
    tail = (_lib.ptr(mask_u8), f32(DL_const).data_ptr(), f32(Ebar).data_ptr(), f32(E).data_ptr(),
            f32(SL1_const).data_ptr(), f32(SL2_const).data_ptr(), const_mode, f32(col_log_probs).data_ptr(),
            int(bool(use_col_weights)), tt.child1.data_ptr(), tt.child2.data_ptr(), tt.parent.data_ptr(),
            tt.jumps.data_ptr(), tt.K, tt.lv_ptr.data_ptr(), tt.n_levels, tt.lv_par.data_ptr(), tt.lv_c1.data_ptr(),
            tt.lv_c2.data_ptr(), int(use_leaf_index), _lib.ptr(i32(leaf_state_idx) if use_leaf_index else None),
            _lib.ptr(f32(leaf_logp) if use_leaf_index else None), leaf_mode, _lib.ptr(leaf_term),
            _lib.ptr(i64(item_idx)))
    n_terms = int(neumann_terms)
    rhs_c = rhs if rhs.stride(1) == 1 else rhs.contiguous()
    if solver == "gmres":
        b = rhs_c.float().reshape(W, S)
        if active_mask is not None:
            b = b * active_mask.reshape(W, -1).to(device=dev, dtype=torch.bool).any(dim=1, keepdim=True).float()
        b = b.contiguous()
        a_out = torch.empty(shape, device=dev, dtype=torch.float32)

        def apply_a(x):
            x = x.contiguous()
            _lib.call("kb_wave_adjoint_apply", *head, *tail, x.data_ptr(), S, a_out.data_ptr(), ws, W, S, st)
            return a_out

        v = _gmres_fixed(apply_a, b, n_terms).contiguous()
        v_k.copy_(v)
        rhs_c, n_terms = v, 0  # the buckets and the column gradient of the solved rows
    _lib.call("kb_wave_adjoint", *head, rhs_c.data_ptr(), int(rhs_c.stride(0)), *tail, n_terms,
              _lib.ptr(initial_v), S, _lib.ptr(grad_col_log_probs), v_k.data_ptr(), aw0.data_ptr(),
              aw1.data_ptr(), aw2.data_ptr(), aw345.data_ptr(), aw3.data_ptr(), aw4.data_ptr(), _lib.ptr(last_rel),
              ws, W, S, st)
    if targets is not None:
        vals, vector = targets
        col_tot = None if vector else torch.empty((2, S), device=dev, dtype=torch.float64)
        _lib.call("kb_wave_adjoint_accum_targets", aw0.data_ptr(), aw1.data_ptr(), aw2.data_ptr(),
                  aw345.data_ptr(), aw3.data_ptr(), aw4.data_ptr(), W, S, vals[0].data_ptr(), vals[1].data_ptr(),
                  int(vector), vals[2].data_ptr(), vals[3].data_ptr(), vals[4].data_ptr(), vals[5].data_ptr(),
                  vals[6].data_ptr(), _lib.ptr(col_tot), st)
    return (*out, last_rel) if return_last_increment else out


def _grad_targets(targets, S: int, device):
    """Validate ``self_loop_grad_targets`` (reference ``wave_backward.py:1615-1625``): seven fp32
    tensors updated in place and the ``param_grad_vector`` flag.  Returns ``(tensors, vector)`` or
    None.  grad_log_pD / grad_log_pS hold ``S`` values with the flag and one without; the other five
    hold ``S``."""
    if targets is None:
        return None
    if len(targets) != 8:
        raise ValueError("self_loop_grad_targets must be (grad_log_pD, grad_log_pS, grad_E, grad_Ebar, "
                         "grad_E_s1, grad_E_s2, grad_mt, param_grad_vector)")
    vals, vector = list(targets[:7]), bool(targets[7])
    for i, t in enumerate(vals):
        need = S if (i >= 2 or vector) else 1
        if not torch.is_tensor(t) or t.device != device or t.dtype != torch.float32 or not t.is_contiguous() \
                or t.numel() < need:
            raise ValueError(f"self_loop_grad_targets[{i}] must be a contiguous fp32 tensor on {device} "
                             f"with at least {need} elements")
    return vals, vector


def _dts_backward_layout(shape, S: int, item_indexed: bool):
    """(row_stride, elem_stride) of a DTS backward parameter or gradient of ``shape``: the value of
    item ``g`` at column ``s`` is at ``g * row_stride + s * elem_stride``; None for a layout the
    reference rejects.  The precedence is the reference's layout contract
    (``kbench/core/kernels/_dts_layout_contract.py:158-200``): one element is a shared scalar; with
    item indexing any 1-D tensor is one value per item (before ``[S]`` is considered); ``[S]`` is
    a shared state row; with item indexing ``[G, 1]`` is one value per item and ``[G, S]`` one row
    per item (one shared row when G = 1)."""
    shape = tuple(int(d) for d in shape)
    n = 1
    for d in shape:
        n *= d
    if n == 1:
        return 0, 0
    if item_indexed and len(shape) == 1:
        return 1, 0
    if len(shape) == 1 and shape[0] == S:
        return 0, 1
    if item_indexed and len(shape) == 2 and shape[1] == 1:
        return 1, 0
    if item_indexed and len(shape) == 2 and shape[1] == S:
        return (0 if shape[0] == 1 else S), 1
    return None


def _param_ref(param, *, S, item_indexed, device):
    """(tensor, row_stride, elem_stride) for the DTS backward parameter layouts
    (reference ``wave_backward.py:103-163``: scalar, [S], [G]/[G,1], [G,S], classified by
    :func:`_dts_backward_layout`)."""
    if not torch.is_tensor(param):
        return torch.tensor([float(param)], device=device, dtype=torch.float32), 0, 0
    lay = _dts_backward_layout(param.shape, S, item_indexed)
    if lay is None:
        raise ValueError("DTS parameters must be scalar, [S], [G], [G, 1], or [G, S] for the fused DTS backward path")
    p = f32(param.to(device)).reshape(-1)
    return p, lay[0], lay[1]


def dts_cross_backward_accum_fused(Pi_star, Pibar_star, v_k, ws, sl, sr, reduce_idx, wlsp, log_pD, log_pS,
                                   node_child1, node_child2, accumulated_rhs, S, active_mask=None,
                                   use_atomics=True, merge_s_term=False, grad_log_pD=None, grad_log_pS=None,
                                   grad_mt=None, accum_param_reductions=False, accum_mt_reduction=False,
                                   output_pibar_ud=False, output_pibar_side_active=False, pibar_side_threshold=0.0,
                                   mt_squeezed=None, pibar_row_max=None, grad_mt_two_stage=False,
                                   grad_mt_two_stage_tile_splits=128, skip_inactive_pibar_output_zero=False,
                                   item_idx=None):
    """Reference ``wave_backward.py:2319-2535``: the adjoint of the split reduction.  Adds each
    split's Pi cotangents into ``accumulated_rhs`` (both children, merged speciation terms),
    stages the Pibar cotangents, and accumulates/returns the parameter cotangents.

    ``use_atomics``, ``merge_s_term`` and ``grad_mt_two_stage*`` select implementation strategies
    in the reference; the result is the same here (one fused kernel)."""
    require_cuda_f32("dts_cross_backward_accum_fused", Pi_star, Pibar_star, v_k, accumulated_rhs)
    S = int(S)
    n = int(sl.shape[0])
    dev = Pi_star.device
    dt = torch.float32
    wlsp_flat = f32(wlsp.squeeze(-1) if wlsp.ndim > 1 else wlsp)
    item_indexed = item_idx is not None
    pD, pD_rs, pD_es = _param_ref(log_pD, S=S, item_indexed=item_indexed, device=dev)
    pS, pS_rs, pS_es = _param_ref(log_pS, S=S, item_indexed=item_indexed, device=dev)
    if (pD_rs, pD_es) != (pS_rs, pS_es):
        raise ValueError("log_pD/log_pS must use the same DTS parameter layout")
    if accum_param_reductions and (grad_log_pD is None or grad_log_pS is None):
        raise ValueError("grad_log_pD/grad_log_pS are required when accumulating DTS scalar reductions")
    if accum_mt_reduction and grad_mt is None:
        raise ValueError("grad_mt is required when accumulating DTS mt reductions")
    if output_pibar_ud and (mt_squeezed is None or pibar_row_max is None):
        raise ValueError("mt_squeezed and pibar_row_max are required when outputting Pibar u_d")
    if output_pibar_side_active and not output_pibar_ud:
        raise ValueError("output_pibar_side_active requires output_pibar_ud")
    thr = float(pibar_side_threshold) if not torch.is_tensor(pibar_side_threshold) else \
        float(pibar_side_threshold.reshape(-1)[0])
    if thr < 0.0:
        raise ValueError("pibar_side_threshold must be non-negative")
    thr_enabled = bool(output_pibar_side_active and (torch.is_tensor(pibar_side_threshold) or thr > 0.0))
    # gradient addressing
    if accum_param_reductions:
        lays = []
        for g in (grad_log_pD, grad_log_pS):
            lay = _dts_backward_layout(g.shape, S, item_indexed)
            if g.dtype != dt or not g.is_contiguous() or lay is None:
                raise ValueError("unsupported DTS gradient layout")
            lays.append(lay)
        if lays[0] != lays[1]:
            raise ValueError("unsupported DTS gradient layout")
        gp_rs, gp_es = lays[0]
    else:
        gp_rs, gp_es = 0, 0
    if accum_mt_reduction:
        if grad_mt.numel() == 1:
            gmt_rs, gmt_es = 0, 0
        elif grad_mt.ndim == 1 and int(grad_mt.shape[0]) == S:
            gmt_rs, gmt_es = 0, 1
        elif item_indexed and grad_mt.ndim == 2 and int(grad_mt.shape[1]) == S:
            gmt_rs, gmt_es = (0 if int(grad_mt.shape[0]) == 1 else S), 1
        else:
            raise ValueError("DTS mt reduction target must be scalar, [S], or [G, S]")
    else:
        gmt_rs, gmt_es = 0, 0
    if output_pibar_ud:
        if mt_squeezed.ndim == 1 and int(mt_squeezed.shape[0]) == S:
            mt_t, mt_rs, mt_es = f32(mt_squeezed), 0, 1
        elif item_indexed and mt_squeezed.ndim == 2 and int(mt_squeezed.shape[1]) == S:
            mt_t = f32(mt_squeezed)
            mt_rs, mt_es = (0 if int(mt_t.shape[0]) == 1 else S), 1
        else:
            raise ValueError("mt_squeezed must have shape [S] or [G, S] when outputting Pibar u_d")
        if pibar_row_max.numel() < Pi_star.shape[0]:
            raise ValueError("pibar_row_max must contain one row-max value per Pi row")
    else:
        mt_t, mt_rs, mt_es = None, 0, 0
    if output_pibar_ud:
        grad_Pibar_l = grad_Pibar_r = None
        pibar_ud = torch.empty((2 * n, S), device=dev, dtype=dt)
        pibar_A = torch.empty((2 * n,), device=dev, dtype=dt)
    else:
        grad_Pibar_l = torch.empty((n, S), device=dev, dtype=dt)
        grad_Pibar_r = torch.empty((n, S), device=dev, dtype=dt)
        pibar_ud = pibar_A = None
    side = torch.empty((2 * n,), device=dev, dtype=torch.bool) if output_pibar_side_active else None
    if accum_param_reductions:
        param_pD = param_pS = None
    else:
        param_pD = torch.empty(n, device=dev, dtype=dt)
        param_pS = torch.empty(n, device=dev, dtype=dt)
    if n:
        _lib.call("kb_dts_adjoint", f32(Pi_star).data_ptr(), f32(Pibar_star).data_ptr(), f32(v_k).data_ptr(),
                  _lib.ptr(u8(active_mask)), i64(sl).data_ptr(), i64(sr).data_ptr(), i64(reduce_idx).data_ptr(),
                  wlsp_flat.data_ptr(), pD.data_ptr(), pD_rs, pD_es, pS.data_ptr(), pS_rs, pS_es,
                  _lib.ptr(i64(item_idx)), i32(node_child1).data_ptr(), i32(node_child2).data_ptr(),
                  accumulated_rhs.data_ptr(), int(bool(output_pibar_ud)), _lib.ptr(pibar_ud), _lib.ptr(pibar_A),
                  _lib.ptr(None if side is None else side.view(torch.uint8)), thr, int(thr_enabled),
                  int(bool(skip_inactive_pibar_output_zero)), _lib.ptr(grad_Pibar_l), _lib.ptr(grad_Pibar_r),
                  int(bool(accum_param_reductions)),
                  _lib.ptr(grad_log_pD if accum_param_reductions else None),
                  _lib.ptr(grad_log_pS if accum_param_reductions else None), gp_rs, gp_es, _lib.ptr(param_pD),
                  _lib.ptr(param_pS), int(bool(accum_mt_reduction)),
                  _lib.ptr(grad_mt if accum_mt_reduction else None), gmt_rs, gmt_es, _lib.ptr(mt_t), mt_rs, mt_es,
                  _lib.ptr(None if pibar_row_max is None else f32(pibar_row_max)), int(ws), n, S,
                  _lib.stream_handle(dev))
    if output_pibar_ud:
        if output_pibar_side_active:
            return pibar_ud, pibar_A, side, param_pD, param_pS
        return pibar_ud, pibar_A, param_pD, param_pS
    return grad_Pibar_l, grad_Pibar_r, param_pD, param_pS


def uniform_cross_pibar_vjp_tree_from_ud_fused(Pi_star, col_log_probs, pibar_ud, pibar_A, sl, sr, accumulated_rhs, S,
                                               active_mask=None, reduce_idx=None, pibar_row_max=None,
                                               skip_zero_sides=False, side_active=None, compact_level_ptr=None,
                                               compact_level_parents=None, compact_level_child1=None,
                                               compact_level_child2=None, grad_col_log_probs=None,
                                               use_col_weights=True, side_active_threshold=0.0):
    """Reference ``wave_backward.py:2748-2896``: per active split side, in-place bottom-up subtree
    sums of ``pibar_ud`` and ``p'_child (A - subtree)`` into the child's adjoint row and
    ``grad_col_log_probs``.  Returns the side-active mask used (or None)."""
    n = int(sl.shape[0])
    if n == 0:
        return None
    require_cuda_f32("uniform_cross_pibar_vjp_tree_from_ud_fused", Pi_star, pibar_ud, accumulated_rhs)
    if active_mask is not None and reduce_idx is None:
        raise ValueError("reduce_idx is required when active_mask is provided")
    if pibar_row_max is None:
        raise ValueError("pibar_row_max is required for DTS-staged Pibar VJP")
    if torch.is_tensor(side_active_threshold):
        if side_active_threshold.numel() != 1:
            raise ValueError("side_active_threshold tensor must contain one value")
        thr_enabled, thr = True, float(side_active_threshold.reshape(-1)[0])
    else:
        thr = float(side_active_threshold)
        if thr < 0.0:
            raise ValueError("side_active_threshold must be non-negative")
        thr_enabled = thr > 0.0
    S = int(S)
    dev = Pi_star.device
    if side_active is not None:
        if side_active.numel() != 2 * n:
            raise ValueError("side_active must have one entry per split side")
        side_active = side_active.contiguous()
    elif skip_zero_sides:
        side_active = torch.empty((2 * n,), device=dev, dtype=torch.bool)
        _lib.call("kb_side_active", pibar_ud.data_ptr(), 2 * n, S, thr, int(thr_enabled),
                  side_active.data_ptr(), _lib.stream_handle(dev))
    if compact_level_ptr is None or compact_level_parents is None or compact_level_child1 is None \
            or compact_level_child2 is None:
        raise ValueError("compact state levels are required for Pibar VJP")
    if compact_level_ptr.numel() < 2:
        raise ValueError("compact_level_ptr must contain at least start and end offsets")
    lv_ptr = i64(compact_level_ptr)
    _lib.call("kb_pibar_vjp_tree", f32(Pi_star).data_ptr(), f32(col_log_probs).data_ptr(),
              int(bool(use_col_weights)), pibar_ud.data_ptr(), f32(pibar_A).data_ptr(),
              _lib.ptr(u8(side_active)), i64(sl).data_ptr(), i64(sr).data_ptr(),
              _lib.ptr(i64(reduce_idx) if reduce_idx is not None else None), _lib.ptr(u8(active_mask)),
              f32(pibar_row_max).data_ptr(), lv_ptr.data_ptr(), int(lv_ptr.numel()) - 1,
              i32(compact_level_parents).data_ptr(), i32(compact_level_child1).data_ptr(),
              i32(compact_level_child2).data_ptr(), accumulated_rhs.data_ptr(), _lib.ptr(grad_col_log_probs), n,
              S, _lib.stream_handle(dev))
    return side_active
