"""E-step wrappers (reference: ``kbench/core/kernels/e_step.py``).

The names ``e_fixed_point_triton``, ``e_step_triton_autograd`` and ``_TritonEStep2D`` are the
reference's (kept so callers bind unchanged); the work runs in the sm_100a kernels of
``csrc/kb_estep.cu`` -- there is no Triton here.
"""

from __future__ import annotations

import torch

from .. import _lib, tree
from ._common import f32, require_cuda_f32, rows_of


def _launch_e_step_forward_2d(E, log_pS_mat, log_pD_mat, log_pL_mat, max_coupling_mat, col_log_probs,
                              node_parent, node_child1, node_child2, max_ancestor_depth, *,
                              max_diff_out=None, out=None, use_col_weights=True):
    """One E application per item row (reference ``e_step.py:244-287``)."""
    require_cuda_f32("_launch_e_step_forward_2d", E)
    G, S = int(E.shape[0]), int(E.shape[1])
    E = f32(E)
    E_new, E_s1, E_s2, Ebar = (torch.empty_like(E) for _ in range(4)) if out is None else out
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    pS, pD, pL, mc = (rows_of(t, G, S) for t in (log_pS_mat, log_pD_mat, log_pL_mat, max_coupling_mat))
    col = f32(col_log_probs.reshape(-1))
    _lib.call("kb_e_step_forward", E.data_ptr(), E_new.data_ptr(), E_s1.data_ptr(), E_s2.data_ptr(),
              Ebar.data_ptr(), _lib.ptr(max_diff_out), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(),
              mc.data_ptr(), col.data_ptr(), tt.parent.data_ptr(), tt.child1.data_ptr(),
              tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K, S, G, int(bool(use_col_weights)),
              _lib.stream_handle(E.device))
    return E_new, E_s1, E_s2, Ebar


class _TritonEStep2D(torch.autograd.Function):
    """Differentiable E application (reference ``e_step.py:290-409``); backward = one fused VJP
    kernel (``kb_e_step_vjp``)."""

    @staticmethod
    def forward(E, log_pS_mat, log_pD_mat, log_pL_mat, max_coupling_mat, col_log_probs, node_parent,
                node_child1, node_child2, max_ancestor_depth, use_col_weights):
        return _launch_e_step_forward_2d(E, log_pS_mat, log_pD_mat, log_pL_mat, max_coupling_mat,
                                         col_log_probs, node_parent, node_child1, node_child2,
                                         int(max_ancestor_depth), use_col_weights=bool(use_col_weights))

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.save_for_backward(inputs[0], *output, *inputs[1:4], inputs[5], *inputs[6:9])
        ctx.max_ancestor_depth = int(inputs[9])
        ctx.use_col_weights = bool(inputs[10])

    @staticmethod
    def backward(ctx, grad_E_new, grad_E_s1_out, grad_E_s2_out, grad_Ebar_out):
        (E, E_new, E_s1, E_s2, Ebar, log_pS_mat, log_pD_mat, log_pL_mat, col_log_probs, node_parent,
         node_child1, node_child2) = ctx.saved_tensors
        grads = e_step_vjp(E, E_new, E_s1, E_s2, Ebar, log_pS_mat, log_pD_mat, log_pL_mat, col_log_probs,
                           node_parent, node_child1, node_child2, ctx.max_ancestor_depth, grad_E_new,
                           grad_E_s1_out, grad_E_s2_out, grad_Ebar_out, use_col_weights=ctx.use_col_weights)
        return (*grads, None, None, None, None, None)


def e_step_vjp(E, E_new, E_s1, E_s2, Ebar, log_pS, log_pD, log_pL, col_log_probs, node_parent, node_child1,
               node_child2, max_ancestor_depth, g_new, g_s1, g_s2, g_ebar, *, use_col_weights=True):
    """The VJP of one E application (``_TritonEStep2D.backward``, reference ``e_step.py:325-409``)
    at saved forward values, as one call: returns (grad_E, grad_pS, grad_pD, grad_pL, grad_mc,
    grad_col); ``g_*`` may be None (zero cotangent)."""
    E = f32(E)
    G, S = int(E.shape[0]), int(E.shape[1])
    tt = tree.tables(node_parent, node_child1, node_child2, int(max_ancestor_depth))
    gs = [None if g is None else f32(g) for g in (g_new, g_s1, g_s2, g_ebar)]
    grad_E, grad_pS, grad_pD, grad_pL, grad_mc = (torch.empty_like(E) for _ in range(5))
    grad_col = torch.empty_like(col_log_probs)
    pS, pD, pL = (rows_of(t, G, S) for t in (log_pS, log_pD, log_pL))
    _lib.call("kb_e_step_vjp", E.data_ptr(), f32(E_new).data_ptr(), f32(E_s1).data_ptr(), f32(E_s2).data_ptr(),
              f32(Ebar).data_ptr(), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), f32(col_log_probs).data_ptr(),
              tt.parent.data_ptr(), tt.child1.data_ptr(), tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K,
              tt.lv_ptr.data_ptr(), tt.n_levels, tt.lv_par.data_ptr(), tt.lv_c1.data_ptr(), tt.lv_c2.data_ptr(),
              *[_lib.ptr(g) for g in gs], grad_E.data_ptr(), grad_pS.data_ptr(), grad_pD.data_ptr(),
              grad_pL.data_ptr(), grad_mc.data_ptr(), grad_col.data_ptr(), S, G, int(bool(use_col_weights)),
              _lib.stream_handle(E.device))
    return grad_E, grad_pS, grad_pD, grad_pL, grad_mc, grad_col


def e_step_triton_autograd(E, log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1,
                           node_child2, max_ancestor_depth, use_col_weights=True):
    """Reference ``e_step.py:412-435``."""
    E_arg = E.contiguous()
    G, S = int(E_arg.shape[0]), int(E_arg.shape[1])
    return _TritonEStep2D.apply(
        E_arg, *(_as_item_state_ad(p, S, G) for p in (log_pS, log_pD, log_pL, max_coupling)),
        col_log_probs.contiguous(), node_parent, node_child1, node_child2, int(max_ancestor_depth),
        bool(use_col_weights))


def _as_item_state_ad(t, S, G):
    """Differentiable [G,S] view of a parameter (autograd flows back through reshape/expand)."""
    if t.ndim == 2 and tuple(t.shape) == (G, S):
        return t.contiguous()
    if t.numel() == S:
        return t.reshape(1, S).expand(G, S).contiguous()
    if t.numel() == G:
        return t.reshape(G, 1).expand(G, S).contiguous()
    return t.reshape(1, 1).expand(G, S).contiguous()


def e_fixed_point_triton(E0, log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1,
                         node_child2, max_ancestor_depth, *, max_iter=2000, tol=1e-8, use_col_weights=True):
    """E fixed point (reference ``e_step.py:438-501``), iterated in one persistent CTA on the
    device (no per-iteration host synchronisation).  Returns (E, E_s1, E_s2, Ebar)."""
    max_iter = int(max_iter)
    tol = float(tol)
    if max_iter < 1:
        raise ValueError("max_iter must be at least 1")
    if tol <= 0.0:
        raise ValueError("tol must be positive")
    require_cuda_f32("e_fixed_point_triton", E0)
    E0 = f32(E0)
    G, S = int(E0.shape[0]), int(E0.shape[1])
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    pS, pD, pL, mc = (rows_of(t, G, S) for t in (log_pS, log_pD, log_pL, max_coupling))
    col = f32(col_log_probs.reshape(-1))
    E_out, E_tmp, E_s1, E_s2, Ebar = (torch.empty_like(E0) for _ in range(5))
    iters = torch.zeros((1,), dtype=torch.int32, device=E0.device)
    _lib.call("kb_e_fixed_point", E0.data_ptr(), E_out.data_ptr(), E_tmp.data_ptr(), E_s1.data_ptr(),
              E_s2.data_ptr(), Ebar.data_ptr(), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), mc.data_ptr(),
              col.data_ptr(), tt.parent.data_ptr(), tt.child1.data_ptr(), tt.child2.data_ptr(),
              tt.jumps.data_ptr(), tt.K, S, G, max_iter, tol, int(bool(use_col_weights)), iters.data_ptr(),
              _lib.stream_handle(E0.device))
    e_fixed_point_triton.last_iters = iters
    return E_out, E_s1, E_s2, Ebar


KB_EADJ_WORK_VECTORS = 17  # include/kb_solver.h


def e_adjoint_solve(E, log_pS, log_pD, log_pL, max_coupling, col_log_probs, node_parent, node_child1,
                    node_child2, max_ancestor_depth, g_E, g_Ebar, g_E_s1, g_E_s2, *, n_fam, max_iter=500,
                    tol=1e-7, breakdown_tol=1e-30, use_col_weights=True, check=True):
    """The E adjoint of ONE shared row (reference ``_implicit_grad.py:373-475``) in one launch:
    ``q = g_E + d/dE[n_fam log2(1 - mean 2^E)] + VJP(g_E_s1, g_E_s2, g_Ebar)``, BiCGSTAB on
    ``(I - J_E^T) w = q`` with the stopping and breakdown rules of ``_implicit_grad.py:28-94``,
    then the E step's parameter cotangents at ``w``.

    Returns ``(w [1,S], grad_params [5,S])`` -- the cotangents of ``(log_pS, log_pD, log_pL,
    max_coupling, col_log_probs)`` through the E step (the Ebar cotangent ``g_Ebar`` included).
    Raises ``RuntimeError`` (the reference's message) when the solve does not converge.  With
    ``check=False`` nothing is read back (no host synchronisation, e.g. inside a CUDA graph): returns
    ``(w, grad_params, status [2] int32, rel [1])`` and :func:`e_adjoint_check` raises later."""
    max_iter, tol, breakdown_tol = int(max_iter), float(tol), float(breakdown_tol)
    if max_iter < 1:
        raise ValueError("max_iter must be at least 1")
    if tol <= 0.0:
        raise ValueError("tol must be positive")
    if breakdown_tol <= 0.0:
        raise ValueError("breakdown_tol must be positive")
    require_cuda_f32("e_adjoint_solve", E)
    S = int(E.shape[-1])
    if E.numel() != S:
        raise ValueError("e_adjoint_solve takes one shared row")
    E = f32(E.reshape(1, S))
    tt = tree.tables(node_parent, node_child1, node_child2, max_ancestor_depth)
    pS, pD, pL, mc = (rows_of(t, 1, S) for t in (log_pS, log_pD, log_pL, max_coupling))
    col = f32(col_log_probs.reshape(-1))
    gs = [f32(g.reshape(1, S)) for g in (g_E, g_Ebar, g_E_s1, g_E_s2)]
    dev = E.device
    work = torch.empty((KB_EADJ_WORK_VECTORS, S), dtype=torch.float32, device=dev)
    w = torch.empty((1, S), dtype=torch.float32, device=dev)
    grad_params = torch.empty((5, S), dtype=torch.float32, device=dev)
    status = torch.zeros((2,), dtype=torch.int32, device=dev)
    rel = torch.zeros((1,), dtype=torch.float32, device=dev)
    _lib.call("kb_e_adjoint_solve", E.data_ptr(), pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), mc.data_ptr(),
              col.data_ptr(), tt.parent.data_ptr(), tt.child1.data_ptr(), tt.child2.data_ptr(),
              tt.jumps.data_ptr(), tt.K, tt.lv_ptr.data_ptr(), tt.n_levels, tt.lv_par.data_ptr(),
              tt.lv_c1.data_ptr(), tt.lv_c2.data_ptr(), *[g.data_ptr() for g in gs], float(n_fam), max_iter,
              tol, breakdown_tol, work.data_ptr(), w.data_ptr(), grad_params.data_ptr(), status.data_ptr(),
              rel.data_ptr(), S, int(bool(use_col_weights)), _lib.stream_handle(dev))
    if not check:
        return w, grad_params, status, rel
    e_adjoint_check(status, rel)
    return w, grad_params


def e_adjoint_check(status, rel):
    """Raise the reference's ``RuntimeError`` when a :func:`e_adjoint_solve` did not converge
    (reads its status words: one host synchronisation)."""
    code, iters = status.tolist()
    e_adjoint_solve.last_iters = iters
    if code != 0:
        raise RuntimeError(f"E-adjoint BiCGSTAB solve failed after {iters} iterations "
                           f"(relative residual {float(rel.item()):.3e})")
