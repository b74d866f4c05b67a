"""Host side of the static builder: the topology sampler and the host layout stage it is checked
against (the device builder's specification), pinned to the generator's output."""

import hashlib

import numpy as np
import pytest

from kbench_b200 import builder, gen

# sha256 (first 16 hex digits) of the generated wave layouts; a change of the generator's output
# changes every fixture made from it
LAYOUT_DIGESTS = {(1, None): "b7a11b0813cf90a9", (4, 3): "9c4d0518f81fff60"}


def layout_digest(static) -> str:
    h = hashlib.sha256()
    wl = static["wave_layout"]
    for k in ("leaf_state_index", "root_row_ids", "item_idx"):
        h.update(np.ascontiguousarray(wl[k]).tobytes())
    for m in wl["wave_metas"]:
        for k in sorted(m):
            h.update(k.encode())
            h.update(np.ascontiguousarray(np.asarray(m[k])).tobytes())
    return h.hexdigest()[:16]


@pytest.mark.parametrize("config,nf", sorted(LAYOUT_DIGESTS, key=str))
def test_generator_layout_pinned(config, nf):
    cap = gen.generate(config, n_families=nf, as_torch=False)
    assert layout_digest(cap["static"]) == LAYOUT_DIGESTS[(config, nf)]


def _trees_ok(topo):
    G = topo["leaf_hash"].shape[1]
    NN = 2 * G - 1
    T = topo["n_topologies"]
    for t in range(topo["left"].shape[0]):
        left, right, root = topo["left"][t], topo["right"][t], int(topo["root"][t])
        assert (left[:G] == -1).all() and (right[:G] == -1).all()
        kids = np.concatenate([left[G:], right[G:]])
        assert ((kids >= 0) & (kids < NN)).all()
        # every node but the root is a child exactly once
        cnt = np.bincount(kids, minlength=NN)
        assert cnt[root] == 0 and (np.delete(cnt, root) == 1).all()
        # the root's clade hash is the sum of the family's leaf hashes
        f = t // T
        h = [0] * NN
        for g in range(G):
            h[g] = int(topo["leaf_hash"][f, g])
        order = []
        stack = [root]
        while stack:
            v = stack.pop()
            order.append(v)
            if v >= G:
                stack += [int(left[v]), int(right[v])]
        for v in reversed(order):
            if v >= G:
                h[v] = (h[left[v]] + h[right[v]]) & gen.MASK64
        assert h[root] == sum(h[:G]) & gen.MASK64


def test_topologies_are_binary_trees():
    species, topo = builder.family_topologies(1)
    assert topo["left"].shape == (8, 2 * 48 - 1) and topo["leaf_hash"].dtype == np.uint64
    _trees_ok(topo)
    assert (topo["leaf_hash"] & np.uint64(1) == 1).all()  # odd: no zero clade hash of one leaf


@pytest.mark.parametrize("config,nf", [(1, None), (4, 3)])
def test_host_reference_is_the_generator(config, nf):
    """The builder's specification (host amalgamation + layout over the stacked topologies) is
    exactly what the generator produces."""
    species, topo = builder.family_topologies(config, n_families=nf)
    static, stats = builder.host_reference(topo, species)
    cap = gen.generate(config, n_families=nf, as_torch=False)
    assert layout_digest(static) == layout_digest(cap["static"])
    for k in ("C", "n_waves", "max_W", "n_splits", "K_children"):
        assert stats[k] == cap["meta"][k]


def test_default_caps_hold_the_instances():
    for T, G in ((8, 48), (16, 512), (64, 4096), (32, 1024)):
        cl, sl = builder.default_caps(T, G)
        assert 2 ** cl >= 1.25 * (T * (G - 1) + G) and 2 ** sl >= 3 * T * (G - 1)


def test_amalgamation_options_change_the_layout():
    """Rounds and smoothing reach the host specification (the device builder is checked against
    these on the GPU)."""
    species, topo = builder.family_topologies(1)
    base, s0 = builder.host_reference(topo, species)
    none, s1 = builder.host_reference(topo, species, amalg_rounds=0)
    assert s1["n_splits"] < s0["n_splits"] and s1["C"] == s0["C"]
    smooth, _ = builder.host_reference(topo, species, alpha=1.5)
    a = np.concatenate([m["log_split_probs"] for m in base["wave_layout"]["wave_metas"] if "sl" in m])
    b = np.concatenate([m["log_split_probs"] for m in smooth["wave_layout"]["wave_metas"] if "sl" in m])
    assert a.shape == b.shape and not np.array_equal(a, b)
