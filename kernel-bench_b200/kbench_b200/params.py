"""Parameter extraction (differentiable torch ops; restates the reference's
``kbench/core/parameters/extract_parameters.py``).

theta[s] = (t_D, t_L, t_T) are log2-odds against speciation: the four event log2-probabilities
of column s are the log2-softmax of (0, t_D, t_L, t_T).
"""

from __future__ import annotations

import math

import torch

LN2 = math.log(2.0)


def as_item_param(t, item_rows, S=None):
    """Reference ``extract_parameters.py:8-15``."""
    if t.ndim == 0:
        return t.reshape(1, 1).expand(int(item_rows), 1).contiguous()
    if t.ndim == 1:
        if S is not None and int(item_rows) == 1 and int(t.numel()) == int(S):
            return t.reshape(1, int(S)).contiguous()
        return t.reshape(int(item_rows), 1).contiguous()
    return t.contiguous()


def as_item_state(t, S, item_rows):
    """Reference ``extract_parameters.py:18-22``."""
    p = as_item_param(t, item_rows, S)
    if int(p.shape[1]) == int(S):
        return p.contiguous()
    return p.expand(int(item_rows), int(S)).contiguous()


def _event_log2p(theta):
    logits = torch.cat((theta.new_zeros((*theta.shape[:-1], 1)), theta), dim=-1)
    return torch.log_softmax(logits * LN2, dim=-1) / LN2


def extract_parameters_uniform(theta, unnorm_row_max, *, statewise=False, itemwise=False):
    """Reference ``extract_parameters.py:25-34`` -> (log_pS, log_pD, log_pL, max_coupling)."""
    r = _event_log2p(theta)
    log_pT = r[..., 3]
    mc = log_pT + unnorm_row_max if (statewise and not itemwise) else log_pT.unsqueeze(-1) + unnorm_row_max
    return r[..., 0], r[..., 1], r[..., 2], mc


def col_log_probs_from_weights(col_weights):
    """Reference ``extract_parameters.py:37-38``: log2 of softmax(col_weights)."""
    return torch.log_softmax(col_weights, dim=-1) / LN2


class _ColValidLogNormalizer(torch.autograd.Function):
    """``col_valid_log_normalizer`` as one kernel each way (``kb_col_normalizer`` and
    ``kb_col_normalizer_vjp``) instead of ``max_ancestor_depth`` rounds of gathers."""

    @staticmethod
    def forward(ctx, col_log_probs, tt, max_ancestor_depth):
        from . import _lib
        clp = col_log_probs.detach().to(torch.float32).contiguous()
        S = int(clp.numel())
        out = torch.empty((S,), dtype=torch.float32, device=clp.device)
        _lib.call("kb_col_normalizer", clp.data_ptr(), tt.parent.data_ptr(), int(max_ancestor_depth), S,
                  out.data_ptr(), _lib.stream_handle(clp.device))
        ctx.save_for_backward(clp)
        ctx.tt = tt
        ctx.depth = int(max_ancestor_depth)
        return out.to(col_log_probs.dtype)

    @staticmethod
    def backward(ctx, g):
        from . import _lib
        (clp,) = ctx.saved_tensors
        tt = ctx.tt
        S = int(clp.numel())
        g = g.detach().to(torch.float32).contiguous()
        grad = torch.empty((S,), dtype=torch.float32, device=clp.device)
        _lib.call("kb_col_normalizer_vjp", clp.data_ptr(), tt.parent.data_ptr(), ctx.depth, _lib.ptr(tt.lv_ptr),
                  tt.n_levels, _lib.ptr(tt.lv_par), _lib.ptr(tt.lv_c1), _lib.ptr(tt.lv_c2), g.data_ptr(),
                  grad.data_ptr(), S, _lib.stream_handle(clp.device))
        return grad, None, None


def col_valid_log_normalizer(col_log_probs, node_parent, max_ancestor_depth, *, tables=None, node_child1=None,
                             node_child2=None):
    """Reference ``extract_parameters.py:41-65``: ``-log2(1 - sum_{anc-or-self} 2^clp)`` (``-inf``
    where the mass reaches 1), differentiable.  One sm_100a kernel each way; the root-path mass is
    summed in the reference's order.  The VJP's subtree sums need the child arrays: pass them, or
    they are derived from ``node_parent`` once per tree."""
    from . import tree
    if not col_log_probs.is_cuda:
        raise RuntimeError("col_valid_log_normalizer runs on the sm_100a kernels: col_log_probs must be on CUDA")
    S = int(col_log_probs.numel())
    tt = tables
    if tt is None:
        if node_child1 is None or node_child2 is None:
            node_child1, node_child2 = tree.children_from_parent(node_parent)
        dev = col_log_probs.device
        tt = tree.tables(node_parent.to(dev), node_child1.to(dev), node_child2.to(dev), int(max_ancestor_depth))
    if tt.S != S:
        raise ValueError(f"node_parent has {tt.S} columns, col_log_probs {S}")
    return _ColValidLogNormalizer.apply(col_log_probs.reshape(S), tt, int(max_ancestor_depth))


def extract_parameters_weighted_cols(theta, col_weights, state_helpers, *, statewise=False, itemwise=False,
                                     uniform_fast=False):
    """Reference ``extract_parameters.py:68-93``."""
    r = _event_log2p(theta)
    log_pT = r[..., 3]
    clp = col_log_probs_from_weights(col_weights.to(device=theta.device, dtype=theta.dtype))
    from . import tree
    sh = state_helpers
    tt = tree.tables(sh["node_parent"], sh["node_child1"], sh["node_child2"], int(sh["max_ancestor_depth"]),
                     compact_level_ptr=sh.get("compact_level_ptr"),
                     compact_level_parents=sh.get("compact_level_parents"),
                     compact_level_child1=sh.get("compact_level_child1"),
                     compact_level_child2=sh.get("compact_level_child2"))
    norm = col_valid_log_normalizer(clp, sh["node_parent"], int(sh["max_ancestor_depth"]), tables=tt)
    mc = log_pT + norm if (statewise and not itemwise) else log_pT.unsqueeze(-1) + norm
    if uniform_fast:
        mc = mc - math.log2(int(state_helpers["S"]))
    return r[..., 0], r[..., 1], r[..., 2], mc, clp
