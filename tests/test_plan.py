"""The dataflow dependency arrays of the engine plan (host side, no GPU): simulating the device
queue on the CPU must release every row exactly once, in an order that respects the splits, for
the forward (children before parents) and the backward (parents before children)."""

import numpy as np
import pytest

from kbench_b200 import engine, gen, runtime


def _simulate(dep, ready, ptr, idx):
    dep = dep.copy()
    order = list(ready)
    i = 0
    while i < len(order):
        r = order[i]
        i += 1
        for j in range(ptr[r], ptr[r + 1]):
            c = idx[j]
            dep[c] -= 1
            assert dep[c] >= 0
            if dep[c] == 0:
                order.append(c)
    return np.asarray(order), dep


@pytest.mark.parametrize("config,seed", [(1, 1000), (2, 2000)])
def test_dataflow_arrays_release_every_row_in_dependency_order(config, seed):
    cap = gen.generate(config, seed=seed)
    static = runtime.make_static(cap, "cpu")
    plan = engine.build_plan(static)
    C = int(cap["meta"]["C"])
    rsp = plan.row_split_ptr.numpy()
    sl, sr = plan.sl_r.numpy(), plan.sr_r.numpy()
    fwd, dep = _simulate(plan.dep0.numpy(), plan.ready0.numpy(), plan.par_ptr.numpy(), plan.par_idx.numpy())
    assert len(fwd) == C and (dep == 0).all() and len(set(fwd.tolist())) == C
    pos = np.empty(C, np.int64)
    pos[fwd] = np.arange(C)
    for p in range(C):
        for n in range(rsp[p], rsp[p + 1]):
            assert pos[sl[n]] < pos[p] and pos[sr[n]] < pos[p]
    bwd, dep = _simulate(plan.dep_b.numpy(), plan.ready_b.numpy(), plan.child_ptr.numpy(), plan.child_idx.numpy())
    assert len(bwd) == C and (dep == 0).all()
    pos[bwd] = np.arange(C)
    for p in range(C):
        for n in range(rsp[p], rsp[p + 1]):
            assert pos[p] < pos[sl[n]] and pos[p] < pos[sr[n]]
    roots = cap["static"]["wave_layout"]["root_row_ids"].numpy()
    assert set(plan.ready_b.numpy().tolist()) == set(roots.tolist())


def test_linear_range_decision():
    """The engine sends every row to the log-space iteration exactly when a finite exponent of
    the linear constants (max(dl, ebar), mc + e, sl1, sl2) is below 2^-26; -inf entries (absent
    terms) do not count."""
    import torch
    from kbench_b200 import engine
    S = 5
    base = {k: torch.full((1, S), -3.0) for k in ("dl", "ebar", "mc", "e", "sl1", "sl2")}
    assert engine.linear_range_ok(base)
    k = dict(base, dl=torch.full((1, S), -40.0))  # hidden by ebar in 2^dl + 2^ebar
    assert engine.linear_range_ok(k)
    k = dict(base, dl=torch.full((1, S), -40.0), ebar=torch.full((1, S), -27.0))
    assert not engine.linear_range_ok(k)
    k = dict(base, mc=torch.full((1, S), -24.0))  # mc + e = -27
    assert not engine.linear_range_ok(k)
    sl = torch.full((1, S), -3.0)
    sl[0, 2] = float("-inf")
    assert engine.linear_range_ok(dict(base, sl1=sl))


@pytest.mark.parametrize("direction", ["forward", "backward"])
def test_start_order_is_topological(direction):
    """The dataflow passes' fixed start orders (kb_list_schedule, host code in the library) put
    every row after the rows it waits for -- children in the forward, parents in the backward: the
    condition under which CTAs taking rows in that order cannot wait on each other forever."""
    from types import SimpleNamespace
    import numpy as np
    from kbench_b200 import engine, gen
    cap = gen.generate(2)
    plan = engine.build_plan(SimpleNamespace(wave_layout=cap["static"]["wave_layout"]))
    order = engine.start_order(plan, direction, 148).numpy()
    C = int(cap["meta"]["C"])
    assert sorted(order.tolist()) == list(range(C))
    pos = np.empty(C, dtype=np.int64)
    pos[order] = np.arange(C)
    cp, ci = plan.child_ptr.numpy(), plan.child_idx.numpy()
    parent_of_pair = np.repeat(np.arange(C), np.diff(cp))  # pairs (row, child)
    if direction == "forward":
        assert (pos[ci] < pos[parent_of_pair]).all()
        assert np.diff(cp)[order[0]] == 0  # the first row started has no children
    else:
        assert (pos[parent_of_pair] < pos[ci]).all()
        assert np.diff(plan.par_ptr.numpy())[order[0]] == 0  # ... no parents


def test_list_schedule_rejects_a_cycle():
    import numpy as np
    from kbench_b200 import _lib
    ptr = np.array([0, 1, 2], dtype=np.int64)
    idx = np.array([1, 0], dtype=np.int32)  # 0 waits for 1 and 1 for 0
    cost = np.ones(2)
    order = np.zeros(2, dtype=np.int32)
    with pytest.raises(ValueError):
        _lib.call("kb_list_schedule", 2, ptr.ctypes.data, idx.ctypes.data, ptr.ctypes.data, idx.ctypes.data,
                  cost.ctypes.data, 4, order.ctypes.data, None)


def test_list_schedule_bounds():
    """The host list scheduler's modelled makespan: the summed cost on one worker, the critical
    path with a worker per row, and in between the classic list-scheduling bounds."""
    from types import SimpleNamespace
    import numpy as np
    from kbench_b200 import _lib, engine, gen
    cap = gen.generate(1)
    plan = engine.build_plan(SimpleNamespace(wave_layout=cap["static"]["wave_layout"]))
    C = int(cap["meta"]["C"])
    cp, ci = plan.child_ptr.numpy().astype(np.int64), plan.child_idx.numpy().astype(np.int32)
    pp, pi = plan.par_ptr.numpy().astype(np.int64), plan.par_idx.numpy().astype(np.int32)
    cost = 1.0 + 0.1 * np.diff(plan.row_split_ptr.numpy()).astype(np.float64)
    # critical path (forward: a row after its children)
    fin = np.zeros(C)
    for r in range(C):  # children have smaller row ids
        fin[r] = cost[r] + (fin[ci[cp[r]:cp[r + 1]]].max() if cp[r + 1] > cp[r] else 0.0)
    crit = fin.max()

    def span(workers):
        order = np.empty(C, dtype=np.int32)
        out = np.zeros(1)
        _lib.call("kb_list_schedule", C, cp.ctypes.data, ci.ctypes.data, pp.ctypes.data, pi.ctypes.data,
                  cost.ctypes.data, workers, order.ctypes.data, out.ctypes.data)
        return float(out[0])

    assert abs(span(1) - cost.sum()) < 1e-6 * cost.sum()
    assert abs(span(C) - crit) < 1e-9 * crit
    for w in (2, 8, 32):
        s = span(w)
        assert max(cost.sum() / w, crit) - 1e-9 <= s <= cost.sum() / w + crit + 1e-9


@pytest.mark.parametrize("config,seed", [(1, 1000), (2, 2000)])
def test_backward_edge_csr_lists_every_split_side_once_in_order(config, seed):
    """The deterministic backward's gather table: each row's incoming edges (edge 2i + side of split
    i, in row-order split numbering) are exactly the split sides that name it as a child, in
    ascending order, and the backward dependency counts (distinct parents) follow from them."""
    import torch
    cap = gen.generate(config, seed=seed)
    static = runtime.make_static(cap, "cpu")
    plan = engine.build_plan(static)
    C, S = int(cap["meta"]["C"]), int(cap["meta"]["S"])
    ed = engine._edge_scratch(static, plan, C, S, torch.device("cpu"))
    assert ed is not None and tuple(ed["rows"].shape) == (2 * plan.n_splits, S)
    ptr, edges = ed["in_ptr"].numpy(), ed["in_edge"].numpy().astype(np.int64)
    assert ptr[0] == 0 and ptr[-1] == 2 * plan.n_splits and (np.diff(ptr) >= 0).all()
    child = np.stack([plan.sl_r.numpy(), plan.sr_r.numpy()], axis=1).reshape(-1)
    rsp = plan.row_split_ptr.numpy()
    parent = np.repeat(np.arange(C), np.diff(rsp))
    for r in range(C):
        e = edges[ptr[r]:ptr[r + 1]]
        assert (np.diff(e) > 0).all() and (child[e] == r).all()
        assert len(set(parent[e // 2].tolist())) == int(plan.dep_b.numpy()[r])
    assert np.array_equal(np.sort(edges), np.arange(2 * plan.n_splits))
    static._deterministic_backward = False
    assert engine._edge_scratch(static, plan, C, S, torch.device("cpu")) is None
