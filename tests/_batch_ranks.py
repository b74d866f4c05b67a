"""Rank bodies for the family-batch tests (imported by spawned processes): the CPU oracle as
the batch's per-chunk solver, and a gloo rank that runs one batch step."""

from __future__ import annotations

import os

import numpy as np
import torch

from kbench_b200 import batch, gen
from oracle import kb_oracle as O

TINY = gen.ProblemConfig("batch-test", 16, 24, 4, 20, 60, n_families=4,
                         solver_options={"e_tol": 1e-6, "e_max_iter": 50, "pi_iters": 6, "neumann_terms": 4})
SEED = 77


def oracle_static(captured):
    st = dict(captured["static"])
    st["solver_options"] = captured["meta"]["solver_options"]
    return st


class OracleSolver:
    """The numpy oracle behind the batch interface (test infrastructure only)."""

    def load(self, captured):
        return oracle_static(captured)

    def prepare(self, static, theta, col_weights):
        return {}

    def new_acc(self, static):
        return torch.zeros((8, int(static["state_helpers"]["S"])), dtype=torch.float64)

    def chunk(self, static, theta, col_weights, prep, acc):
        loss, saved = O.forward(static, theta, col_weights)
        a = O.backward_accumulators(static, saved)
        acc += torch.from_numpy(np.stack([a[n] for n in batch.ACC_NAMES]).astype(np.float64))
        prep["saved"] = saved
        return torch.tensor(loss, dtype=torch.float64)

    def reduce_acc(self, acc, S):
        return acc

    def finish(self, static, theta, col_weights, prep, acc8, n_fam):
        a = {n: acc8[j].numpy().astype(np.float32) for j, n in enumerate(batch.ACC_NAMES)}
        return O.e_adjoint_and_theta_vjp(static, theta, col_weights, prep["saved"], O.Tree(static["state_helpers"]),
                                         a["E"], a["Ebar"], a["E_s1"], a["E_s2"], a["pD"], a["pS"], a["mt"],
                                         a["col"], n_fam=n_fam)


class EngineOnCpuSolver(batch.EngineSolver):
    """The engine's batch solver with only its device steps replaced: ``load`` is the engine's own
    (``runtime.make_static`` + ``engine.build_plan`` on the host), the column sums go into the
    engine's fp64 slot layout ``[n_slots, 8, NTV]`` and are combined by the engine's
    ``reduce_acc``; the forward + accumulating backward of a chunk, ``prepare`` and ``finish`` (CUDA
    kernels) are computed by the oracle instead."""

    N_SLOTS = 3

    def __init__(self):
        super().__init__("cpu")
        self._next_slot = 0

    def load(self, captured):
        static = super().load(captured)
        static._oracle_static = oracle_static(captured)
        return static

    def prepare(self, static, theta, col_weights):
        return {}

    def new_acc(self, static):
        from kbench_b200 import tree
        bd, vpt = tree.engine_width(int(static.state_helpers["S"]))
        return torch.zeros((self.N_SLOTS, 8, bd * vpt), dtype=torch.float64)

    def chunk(self, static, theta, col_weights, prep, acc):
        st = static._oracle_static
        loss, saved = O.forward(st, theta, col_weights)
        a = O.backward_accumulators(st, saved)
        S = int(st["state_helpers"]["S"])
        slot = self._next_slot % self.N_SLOTS  # a CTA's slot: chunks spread over several
        self._next_slot += 1
        acc[slot, :, :S] += torch.from_numpy(np.stack([a[n] for n in batch.ACC_NAMES]).astype(np.float64))
        prep["saved"], prep["static"] = saved, st
        return torch.tensor(loss, dtype=torch.float64)

    def finish(self, static, theta, col_weights, prep, acc8, n_fam):
        return OracleSolver().finish(prep["static"], theta, col_weights, prep, acc8, n_fam)


SOLVERS = {"oracle": OracleSolver, "engine_cpu": EngineOnCpuSolver}


def gloo_rank(rank, world, port, chunk, out_dir, solver="oracle"):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n = TINY.n_families
        f0, f1 = batch.family_block(n, world, rank)
        chunks = batch.build_chunks(TINY, f0, f1, chunk, seed=SEED, workers=1)
        fb = batch.FamilyBatch(chunks, n, SOLVERS[solver](), allreduce=lambda t: dist.all_reduce(t))
        theta = chunks[0]["inputs"]["theta"]
        col = chunks[0]["inputs"]["col_weights"]
        res = fb.step(theta, col)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), loss=float(res.loss), grad_theta=res.grad_theta,
                 grad_col=res.grad_col, f0=f0, f1=f1, n_chunks=len(chunks))
    finally:
        dist.destroy_process_group()
