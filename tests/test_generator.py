"""Invariants of the synthetic problem layout (the contract the reference kernels assume)."""

import numpy as np
import pytest

from kbench_b200 import engine, gen, tree


@pytest.fixture(scope="module")
def small():
    return gen.generate(1, as_torch=False)


def test_species_tree(small):
    sh = small["static"]["state_helpers"]
    S = sh["S"]
    par, c1, c2 = sh["node_parent"], sh["node_child1"], sh["node_child2"]
    assert S == 2 * 32 - 1
    assert (par == -1).sum() == 1 and par[S - 1] == -1  # postorder: root last
    internal = c1 < S
    assert (c1[~internal] == S).all() and (c2[~internal] == S).all()  # leaf sentinel S
    assert (c1[internal] < np.nonzero(internal)[0]).all()  # children before parents
    for x in np.nonzero(internal)[0]:
        assert par[c1[x]] == x and par[c2[x]] == x
    st, en = sh["node_subtree_start"], sh["node_subtree_end"]
    assert sorted(st.tolist()) == list(range(S))  # preorder permutation
    for x in np.nonzero(internal)[0]:
        assert st[x] < st[c1[x]] < en[x] and st[x] < st[c2[x]] < en[x]
    depth = np.zeros(S, int)
    for s in range(S - 1, -1, -1):
        if par[s] >= 0:
            depth[s] = depth[par[s]] + 1
    assert sh["max_ancestor_depth"] == depth.max() + 1
    np.testing.assert_allclose(sh["unnorm_row_max"], -np.log2(S - (depth + 1)), rtol=1e-6)
    ptr = sh["compact_level_ptr"]
    seen = set()
    for lv in range(len(ptr) - 1):  # bottom-up valid: children processed in earlier levels
        nodes = sh["compact_level_parents"][ptr[lv]:ptr[lv + 1]]
        for p in nodes:
            for c in (c1[p], c2[p]):
                assert c >= S or c not in internal.nonzero()[0] or c in seen
        seen.update(nodes.tolist())


def test_waves_and_splits(small):
    wl = small["static"]["wave_layout"]
    C = small["meta"]["C"]
    assert abs(C - 300) / 300 < 0.1
    metas = wl["wave_metas"]
    assert "sl" not in metas[0] and metas[0]["start"] == 0
    assert (wl["leaf_state_index"][: metas[0]["W"]] >= 0).all()
    covered = 0
    for m in metas:
        assert m["start"] == covered
        covered += m["W"]
        if "sl" not in m:
            continue
        ws = m["start"]
        assert (m["sl"] < ws).all() and (m["sr"] < ws).all()  # children in earlier waves
        red = m["reduce_idx"]
        n_eq1 = m["n_eq1"]
        assert (np.diff(red[:n_eq1]) > 0).all() or n_eq1 <= 1
        ptr = m["ge2_ptr"]
        assert ptr[0] == 0 and ptr[-1] == len(red) - n_eq1
        for g, p in enumerate(m["ge2_parent_ids"]):
            assert (red[n_eq1 + ptr[g]:n_eq1 + ptr[g + 1]] == p).all() and ptr[g + 1] - ptr[g] >= 2
        assert set(red.tolist()) == set(range(m["W"]))  # every parent has a split
        assert (m["log_split_probs"] <= 0).all()
    assert covered == C


def test_level_plan_is_a_valid_schedule(small):
    import types
    cap = gen.to_torch(small)
    st = types.SimpleNamespace(wave_layout=cap["static"]["wave_layout"])
    plan = engine.build_plan(st)
    lvl = plan.level_of
    rows = plan.rows.numpy()
    sp = plan.split_ptr.numpy()
    sl, sr = plan.sl.numpy(), plan.sr.numpy()
    for i, r in enumerate(rows):
        for j in range(sp[i], sp[i + 1]):
            assert lvl[sl[j]] < lvl[r] and lvl[sr[j]] < lvl[r]
    assert sp[-1] == small["meta"]["n_splits"]
    assert plan.n_levels < len(small["static"]["wave_layout"]["wave_metas"])


def test_packed_column_tables(small):
    sh = small["static"]["state_helpers"]
    S = sh["S"]
    bd, vpt = tree.engine_width(S)
    ntv = bd * vpt
    pk = tree.pack_columns(sh["node_parent"], sh["node_child1"], sh["node_child2"], sh["node_subtree_start"],
                           sh["node_subtree_end"], ntv=ntv).view(np.uint32)
    tour = np.concatenate([pk[1] & 0xFFFF, pk[1] >> 16])
    assert sorted(tour.tolist()) == list(range(2 * ntv))
    rng = np.random.default_rng(1)
    P = np.concatenate([rng.random(S), np.zeros(ntv - S)])
    T = np.zeros(2 * ntv)
    T[pk[1] & 0xFFFF] += P
    T[pk[1] >> 16] -= P
    path = np.cumsum(T)[pk[1] & 0xFFFF]
    for x in range(S):
        want, c = 0.0, x
        while c >= 0:
            want += P[c]
            c = sh["node_parent"][c]
        assert abs(path[x] - want) < 1e-9
    # row 4, by preorder position: subtree end and the parent's position of the column there
    pre, end, par = pk[2] & 0xFFFF, pk[2] >> 16, pk[3] & 0xFFFF
    assert sorted(pre.tolist()) == list(range(ntv))
    assert pk.shape[0] == 5
    for x in range(ntv):
        q = int(pre[x])
        assert int(pk[4][q] & 0xFFFF) == int(end[x])
        assert int(pk[4][q] >> 16) == int(pre[par[x]])
    # the subtree sums the Neumann sweep takes from a prefix over positions match a direct sum
    w = np.concatenate([rng.random(S), np.zeros(ntv - S)])
    xq = np.zeros(ntv)
    xq[pre] = w
    excl = np.concatenate([[0.0], np.cumsum(xq)])
    for x in range(S):
        want, stack = 0.0, [x]
        while stack:
            c = stack.pop()
            want += w[c]
            stack += [k for k in (sh["node_child1"][c], sh["node_child2"][c]) if 0 <= k < S]
        q = int(pre[x])
        assert abs(excl[int(pk[4][q] & 0xFFFF)] - excl[q] - want) < 1e-9
