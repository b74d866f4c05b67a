"""Placeholder until the fused engine lands: delegates to the reference-structured driver."""

from . import glue


def forward(static, theta, col_weights):
    return glue.solve_e_pi(static, theta, col_weights)


def backward(static, theta, col_weights, saved):
    return glue.implicit_grad(static, theta, col_weights, saved)
