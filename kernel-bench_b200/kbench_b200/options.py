"""Solver options (same fields, defaults and validation errors as the reference's
``kbench/api/solver_options.py:4-43``)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class SolverOptions:
    e_init: float = -1.0
    e_max_iter: int = 2000
    e_tol: float = 1e-8
    pi_iters: int = 6
    neumann_terms: int = 3
    self_loop_solver: str = "neumann"
    bicgstab_max_iter: int = 500
    bicgstab_tol: float = 1e-7
    bicgstab_breakdown_tol: float = 1e-30
    adjoint_pruning_threshold: float = 1e-6
    use_adjoint_pruning: bool = True
    pibar_side_threshold: float = 0.0

    def validate(self) -> None:
        checks = (
            (int(self.e_max_iter) >= 1, "e_max_iter must be at least 1"),
            (float(self.e_tol) > 0.0, "e_tol must be positive"),
            (int(self.pi_iters) >= 2 and int(self.pi_iters) % 2 == 0, "pi_iters must be an even integer at least 2"),
            (int(self.neumann_terms) >= 0, "neumann_terms must be non-negative"),
        )
        for ok, msg in checks:
            if not ok:
                raise ValueError(msg)
        solver = str(self.self_loop_solver).strip().lower()
        if solver not in ("neumann", "gmres"):
            raise ValueError("self_loop_solver must be one of: neumann, gmres")
        self.self_loop_solver = solver
        for ok, msg in (
            (int(self.bicgstab_max_iter) >= 1, "bicgstab_max_iter must be at least 1"),
            (float(self.bicgstab_tol) > 0.0, "bicgstab_tol must be positive"),
            (float(self.bicgstab_breakdown_tol) > 0.0, "bicgstab_breakdown_tol must be positive"),
            (float(self.adjoint_pruning_threshold) >= 0.0, "adjoint_pruning_threshold must be non-negative"),
            (float(self.pibar_side_threshold) >= 0.0, "pibar_side_threshold must be non-negative"),
        ):
            if not ok:
                raise ValueError(msg)
