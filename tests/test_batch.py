"""Family batches (the batched config): sharding, chunking, the packed all-reduce, and the
combined result against one oracle run over all the families.  The multi-rank case runs as two
gloo ranks on the CPU with the numpy oracle as the per-chunk solver."""

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as tmp

from _batch_ranks import SEED, TINY, OracleSolver, gloo_rank, oracle_static
from _util import assert_close, assert_loss
from kbench_b200 import batch, gen
from oracle import kb_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _whole_batch_reference():
    cap = gen.generate(TINY, seed=SEED, as_torch=False)
    st = oracle_static(cap)
    loss, saved = O.forward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"])
    gt, gc = O.backward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"], saved)
    return loss, gt, gc


@pytest.mark.parametrize("n,world", [(1024, 1), (1024, 8), (10, 3), (2, 4), (0, 2)])
def test_family_blocks_partition(n, world):
    blocks = [batch.family_block(n, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == n
    for (a0, a1), (b0, b1) in zip(blocks, blocks[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1


def test_chunk_ranges_and_errors():
    assert batch.chunk_ranges(3, 10, 4) == [(3, 7), (7, 10)]
    assert batch.chunk_ranges(5, 5, 4) == []
    with pytest.raises(ValueError):
        batch.chunk_ranges(0, 4, 0)
    with pytest.raises(ValueError):
        batch.family_block(4, 2, 2)


def test_pack_roundtrip():
    S = 7
    loss = torch.tensor(3.5, dtype=torch.float32)
    acc = torch.arange(8 * S, dtype=torch.float64).view(8, S)
    p = batch.pack(loss, acc)
    l2, a2 = batch.unpack(p, S)
    assert float(l2[0]) == 3.5 and torch.equal(a2, acc)
    with pytest.raises(ValueError):
        batch.unpack(p[:-1], S)


def test_chunks_are_slices_of_the_whole_batch():
    """A chunk's families are generated from the same seeds as in the whole-batch generator."""
    whole = gen.generate(TINY, seed=SEED, as_torch=False)
    parts = batch.build_chunks(TINY, 0, TINY.n_families, 2, seed=SEED, workers=1)
    assert [p["meta"]["n_items"] for p in parts] == [2, 2]
    assert sum(p["meta"]["C"] for p in parts) == whole["meta"]["C"]
    np.testing.assert_array_equal(parts[0]["inputs"]["theta"], whole["inputs"]["theta"])


@pytest.mark.parametrize("chunk", [1, 3])
def test_single_rank_chunked_matches_whole_batch(chunk):
    loss_ref, gt_ref, gc_ref = _whole_batch_reference()
    chunks = batch.build_chunks(TINY, 0, TINY.n_families, chunk, seed=SEED, workers=1)
    fb = batch.FamilyBatch(chunks, TINY.n_families, OracleSolver())
    res = fb.step(chunks[0]["inputs"]["theta"], chunks[0]["inputs"]["col_weights"])
    assert_loss(float(res.loss), loss_ref)
    assert_close("grad_theta", res.grad_theta, gt_ref)
    assert_close("grad_col", res.grad_col, gc_ref)


def test_two_gloo_ranks_match_whole_batch(tmp_path):
    loss_ref, gt_ref, gc_ref = _whole_batch_reference()
    world = 2
    tmp.spawn(gloo_rank, args=(world, _free_port(), 1, str(tmp_path)), nprocs=world, join=True)
    outs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    assert [int(o["f1"]) - int(o["f0"]) for o in outs] == [2, 2]
    for o in outs:
        assert_loss(float(o["loss"]), loss_ref)
        assert_close("grad_theta", o["grad_theta"], gt_ref)
        assert_close("grad_col", o["grad_col"], gc_ref)
    np.testing.assert_array_equal(outs[0]["grad_theta"], outs[1]["grad_theta"])


def test_two_gloo_ranks_engine_solver_match_whole_batch(tmp_path):
    """The rank loop over the engine's own batch solver (host-side static and plan building, fp64
    slot layout and slot reduction; only the device steps computed by the oracle) on two gloo
    ranks gives the whole-batch result."""
    loss_ref, gt_ref, gc_ref = _whole_batch_reference()
    world = 2
    tmp.spawn(gloo_rank, args=(world, _free_port(), 1, str(tmp_path), "engine_cpu"), nprocs=world, join=True)
    outs = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for o in outs:
        assert_loss(float(o["loss"]), loss_ref)
        assert_close("grad_theta", o["grad_theta"], gt_ref)
        assert_close("grad_col", o["grad_col"], gc_ref)
    np.testing.assert_array_equal(outs[0]["grad_theta"], outs[1]["grad_theta"])
