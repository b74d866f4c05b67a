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


def col_valid_log_normalizer(col_log_probs, node_parent, max_ancestor_depth):
    """Reference ``extract_parameters.py:41-65``: ``-log2(1 - sum_{anc-or-self} 2^clp)``."""
    S = int(col_log_probs.numel())
    probs = torch.exp2(col_log_probs)
    parent = node_parent.to(device=col_log_probs.device, dtype=torch.long)
    cur = torch.arange(S, device=col_log_probs.device, dtype=torch.long)
    mass = torch.zeros((S,), device=col_log_probs.device, dtype=col_log_probs.dtype)
    zero = mass.new_zeros(())
    for _ in range(max(1, int(max_ancestor_depth))):
        valid = (cur >= 0) & (cur < S)
        safe = cur.clamp(0, max(S - 1, 0))
        mass = mass + torch.where(valid, probs.index_select(0, safe), zero)
        cur = torch.where(valid, parent.index_select(0, safe), torch.full_like(cur, -1))
    vm = 1.0 - mass
    return torch.where(vm > 0.0, -torch.log2(vm.clamp_min(torch.finfo(col_log_probs.dtype).tiny)),
                       col_log_probs.new_full((S,), float("-inf")))


def extract_parameters_weighted_cols(theta, col_weights, state_helpers, *, statewise=False, itemwise=False,
                                     uniform_fast=False):
    """Reference ``extract_parameters.py:68-93``."""
    r = _event_log2p(theta)
    log_pT = r[..., 3]
    clp = col_log_probs_from_weights(col_weights.to(device=theta.device, dtype=theta.dtype))
    norm = col_valid_log_normalizer(clp, state_helpers["node_parent"], int(state_helpers["max_ancestor_depth"]))
    mc = log_pT + norm if (statewise and not itemwise) else log_pT.unsqueeze(-1) + norm
    if uniform_fast:
        mc = mc - math.log2(int(state_helpers["S"]))
    return r[..., 0], r[..., 1], r[..., 2], mc, clp
