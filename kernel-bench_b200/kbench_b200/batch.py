"""Family batches: many gene families sharing one species tree and one theta (the benchmark's
batched workload), processed in memory-bounded chunks on one GPU and sharded across ranks.

Families are independent given theta.  The loss is a sum over families (``solver.py:132-142``
sums the per-root NLL), and every accumulator of the backward (the parameter cotangents, the
E / Ebar / E_s1 / E_s2 cotangents and the column sum, ``_implicit_grad.py:144-158``) is a sum
over rows.  The E fixed point depends on theta only (``solver.py:45``), and the E adjoint and
theta VJP (``_implicit_grad.py:373-475``) are applied once to the summed accumulators.  So:

* each rank takes a contiguous block of the families (:func:`family_block`);
* it runs the fused engine over its block chunk by chunk (:func:`chunk_ranges`), every chunk
  adding its column sums into ONE set of fp64 accumulators on the device;
* ONE all-reduce (sum) of the packed ``[loss, 8 x S accumulators]`` combines the ranks;
* every rank applies the E adjoint and theta VJP to the summed accumulators (S-sized work) and
  holds the same ``(loss, grad_theta, grad_col)``.

This is the computation the reference performs over one static holding all the families; only
the order of the fp64 row sums differs.  The solver is pluggable (:class:`EngineSolver` on the
GPU) so the host-side logic can be driven by other backends.
"""

from __future__ import annotations

import multiprocessing as mp
import os
from dataclasses import dataclass

import torch

from . import gen

ACC_NAMES = ("pD", "pS", "mt", "E", "Ebar", "E_s1", "E_s2", "col")


def family_block(n_families: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block ``[f0, f1)`` of ``n_families`` owned by ``rank`` of ``world`` (the first
    ``n_families % world`` ranks take one extra family)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_families < 0:
        raise ValueError("n_families must be >= 0")
    base, extra = divmod(n_families, world)
    f0 = rank * base + min(rank, extra)
    return f0, f0 + base + (1 if rank < extra else 0)


def chunk_ranges(f0: int, f1: int, chunk: int) -> list[tuple[int, int]]:
    """``[f0, f1)`` cut into consecutive chunks of at most ``chunk`` families."""
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    return [(a, min(a + chunk, f1)) for a in range(f0, f1, chunk)]


def pack(loss, acc8):
    """``[1 + 8*S]`` float64 vector: the loss, then the 8 accumulator rows (``ACC_NAMES``)."""
    return torch.cat([loss.reshape(1).to(torch.float64), acc8.to(torch.float64).reshape(-1)])


def unpack(packed, S: int):
    """Inverse of :func:`pack`: ``(loss [1], acc8 [8,S])``."""
    if packed.numel() != 1 + 8 * S:
        raise ValueError(f"packed vector has {packed.numel()} entries, expected {1 + 8 * S}")
    return packed[:1], packed[1:].view(8, S)


def _build_unit(args):
    config, seed, offset, n, solver_options = args
    return gen.generate(config, seed=seed, n_families=n, family_offset=offset, as_torch=False,
                        solver_options=solver_options)


def build_chunks(config, f0: int, f1: int, chunk: int, *, seed: int | None = None, workers: int | None = None,
                 solver_options: dict | None = None) -> list[dict]:
    """The ``captured`` dicts (numpy) of families ``[f0, f1)`` of a batched config, one per chunk
    of at most ``chunk`` families; family ``f`` is generated from seed ``seed + 1 + f`` exactly as
    :func:`gen.generate` would over the whole batch.  Chunks are built by a ``spawn`` process
    pool (safe after CUDA is initialised) of ``workers`` processes (default: the CPUs this
    process may use)."""
    cfg_id = config if isinstance(config, int) else 0
    seed = 1000 * cfg_id if seed is None else int(seed)
    jobs = [(config, seed, a, b - a, solver_options) for a, b in chunk_ranges(f0, f1, chunk)]
    if workers is None:
        workers = len(os.sched_getaffinity(0))
    workers = max(1, min(int(workers), len(jobs)))
    if workers == 1:
        return [_build_unit(j) for j in jobs]
    with mp.get_context("spawn").Pool(workers) as pool:
        return pool.map(_build_unit, jobs, chunksize=1)


class EngineSolver:
    """The fused B200 engine as the batch's per-chunk solver."""

    def __init__(self, device):
        self.device = torch.device(device)

    def load(self, captured):
        from . import engine, runtime
        static = runtime.make_static(captured, self.device)
        if not engine.supported(static) or static.solver_options.self_loop_solver != "neumann":
            raise ValueError("family batches need the fused engine's layout (statewise, shared theta, Neumann)")
        engine.build_plan(static)
        return static

    def prepare(self, static, theta, col_weights):
        from . import engine
        return engine.prepare(static, theta, col_weights)

    def new_acc(self, static):
        from . import engine
        return engine.new_grad_slots(static, self.device)

    def chunk(self, static, theta, col_weights, prep, acc):
        """Forward + accumulating backward of one chunk; returns its loss (device scalar)."""
        from . import engine, glue, runtime
        out, extras = engine.forward(static, theta, col_weights, prep=prep, check_errors=False)
        loss = glue.nll_from_root_rows(out[4], out[0])
        saved = dict(zip(runtime.FORWARD_SAVED_NAMES, out))
        saved.update(extras)
        engine.backward(static, theta, col_weights, saved, slots=acc, finish=False)
        return loss

    def reduce_acc(self, acc, S):
        return acc.sum(dim=0)[:, :S]

    def check(self, static):
        """Raise if a chunk's dataflow launches gave up a wait (one host synchronisation)."""
        from . import engine
        engine.check_flow_errors(static)

    def finish(self, static, theta, col_weights, prep, acc8, n_fam):
        from . import engine, glue
        S = int(static.state_helpers["S"])
        g = engine.grad_accumulators_from(prep.E, S, acc8.to(torch.float32))
        saved = {"E": prep.E, "E_s1": prep.E_s1, "E_s2": prep.E_s2, "Ebar": prep.Ebar, "log_pS": prep.pS,
                 "log_pD": prep.pD, "log_pL": prep.pL, "max_coupling": prep.mc, "col_log_probs": prep.clp}
        # convergence read back by check() at the end of the step
        return glue.e_adjoint_and_theta_vjp(static, theta, col_weights, saved, g, n_fam, prep.ucw, check=False)


@dataclass
class StepResult:
    loss: torch.Tensor        # float64 scalar: sum over ALL families (every rank)
    grad_theta: torch.Tensor
    grad_col: torch.Tensor


class FamilyBatch:
    """One rank's share of a family batch: ``chunks`` (captured dicts) are loaded by ``solver``;
    :meth:`step` runs forward + backward over them and combines the ranks with one all-reduce.

    ``allreduce(t)`` sums a tensor in place over the ranks (``torch.distributed.all_reduce``;
    ``None`` on a single rank); ``n_total_families`` is the batch size over all ranks."""

    def __init__(self, chunks, n_total_families: int, solver, *, allreduce=None):
        if not chunks:
            raise ValueError("a rank needs at least one chunk of families")
        self.solver = solver
        self.statics = [solver.load(c) for c in chunks]
        self.n_total = int(n_total_families)
        self.allreduce = allreduce
        self.n_local = sum(int(c["meta"]["n_items"]) for c in chunks)
        self.rows = sum(int(c["meta"]["C"]) for c in chunks)

    def step(self, theta, col_weights) -> StepResult:
        s0 = self.statics[0]
        S = int(s0.state_helpers["S"]) if hasattr(s0, "state_helpers") else int(s0["state_helpers"]["S"])
        prep = self.solver.prepare(s0, theta, col_weights)
        acc = self.solver.new_acc(s0)
        loss = None
        for static in self.statics:
            lc = self.solver.chunk(static, theta, col_weights, prep, acc).to(torch.float64)
            loss = lc if loss is None else loss + lc
        packed = pack(loss, self.solver.reduce_acc(acc, S))
        if self.allreduce is not None:
            self.allreduce(packed)
        loss_t, acc8 = unpack(packed, S)
        grad_theta, grad_col = self.solver.finish(s0, theta, col_weights, prep, acc8, self.n_total)
        check = getattr(self.solver, "check", None)
        if check is not None:  # after the whole step is enqueued
            for static in self.statics:
                check(static)
        return StepResult(loss_t[0], grad_theta, grad_col)
