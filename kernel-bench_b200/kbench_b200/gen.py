"""Seeded synthetic problem generator (the static layout the solver consumes).

The reference ships no fixtures (its ``fixtures/*.pt`` and ``data/`` are git-ignored and the
preprocessing that produced them is not in the project, ``capture/capture.py:17-18``), so this
module builds the same ``captured`` dictionary that ``kbench/runtime.py:47-60`` (``make_static``)
consumes, from the textual configs of the benchmark:

* species tree: uniform random pairwise merges of ``n`` leaves -> ``S = 2n-1`` columns, numbered
  in postorder (children before parents, root last);
* gene side: ``T`` gene-tree topologies over ``G`` gene leaves (one random base topology plus
  ``T-1`` copies perturbed by random nearest-neighbour interchanges), each gene leaf mapped to a
  uniformly drawn species leaf;
* rows: the union of all clades seen in the topologies; a row's splits are the bipartitions
  observed for it, plus the bipartitions one rearrangement away whose two parts are both rows
  (amalgamation); the split weight is the smoothed conditional split frequency in log2;
* waves: rows grouped by clade size, smallest first (the leaf wave first, without split keys).

Layout conventions follow the reference kernels: leaf child sentinel is ``S``
(``wave_step.py:920-924``), ``node_subtree_start/end`` is the preorder interval used by the
leaf-seed descendant test (``wave_step.py:1024-1028``), ``unnorm_row_max[s] = -log2(S - #anc-or-
self(s))`` so the uniform forward (``extract_parameters.py:25-34``) agrees with the weighted
backward, compact levels list internal nodes deepest level first (``wave_backward.py:479-512``
pristine), and the split arrays of a wave hold the single-split parents first, then the
multi-split parents grouped by parent (``dts_fused.py:86-97,199-230``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

_U64 = np.uint64
MASK64 = (1 << 64) - 1


@dataclass(frozen=True)
class ProblemConfig:
    name: str
    n_species: int          # species leaves (S = 2n-1)
    n_genes: int            # gene leaves per family
    n_topologies: int       # gene-tree topologies per family
    spr_moves: int          # rearrangement moves applied to each perturbed copy
    target_C: int           # rows per family the config text asks for (reported, not enforced)
    n_families: int = 1
    solver_options: dict = field(default_factory=lambda: {
        "e_tol": 1e-6, "e_max_iter": 50, "pi_iters": 16, "neumann_terms": 16,
    })


# The benchmark's five configurations.  ``spr_moves`` was chosen so the clade union lands within
# about 10% of the row count each config names; the achieved counts are recorded in ``meta``.
CONFIGS = {
    1: ProblemConfig("small", 32, 48, 8, 80, 300),
    2: ProblemConfig("medium", 256, 512, 16, 3200, 8192),
    3: ProblemConfig("large", 2048, 4096, 64, 7500, 131072),
    4: ProblemConfig("batched", 512, 1024, 32, 1350, 16384, n_families=1024),
    5: ProblemConfig("tangent", 2048, 4096, 64, 7500, 131072),
}


# ----------------------------------------------------------------------------------------------
# species tree
# ----------------------------------------------------------------------------------------------

def _random_merge_tree(n_leaves: int, rng: np.random.Generator):
    """Binary tree by uniform random pairwise merges. Nodes 0..n-1 leaves, n..2n-2 internal."""
    n_nodes = 2 * n_leaves - 1
    left = np.full(n_nodes, -1, dtype=np.int64)
    right = np.full(n_nodes, -1, dtype=np.int64)
    parent = np.full(n_nodes, -1, dtype=np.int64)
    active = list(range(n_leaves))
    nxt = n_leaves
    draws = rng.random(2 * n_leaves)
    k = 0
    while len(active) > 1:
        m = len(active)
        i = int(draws[k] * m); k += 1
        j = int(draws[k] * (m - 1)); k += 1
        if j >= i:
            j += 1
        a, b = active[i], active[j]
        left[nxt], right[nxt] = a, b
        parent[a] = parent[b] = nxt
        # remove i and j (swap-remove, larger index first)
        for idx in sorted((i, j), reverse=True):
            active[idx] = active[-1]
            active.pop()
        active.append(nxt)
        nxt += 1
    return left, right, parent, active[0]


def make_species_tree(n_leaves: int, seed: int) -> dict:
    """Species tree with columns in postorder; returns the ``state_helpers`` arrays (numpy)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    left, right, parent, root = _random_merge_tree(n_leaves, rng)
    S = 2 * n_leaves - 1
    # postorder numbering (left subtree, right subtree, node)
    post = np.empty(S, dtype=np.int64)
    pre = np.empty(S, dtype=np.int64)
    size = np.ones(S, dtype=np.int64)
    order = []
    stack = [(root, False)]
    pre_counter = 0
    while stack:
        node, done = stack.pop()
        if done:
            order.append(node)
            continue
        pre[node] = pre_counter
        pre_counter += 1
        stack.append((node, True))
        if left[node] >= 0:
            stack.append((right[node], False))
            stack.append((left[node], False))
    for idx, node in enumerate(order):
        post[node] = idx
    for node in order:
        if left[node] >= 0:
            size[node] = 1 + size[left[node]] + size[right[node]]
    # relabel to postorder ids
    node_parent = np.full(S, -1, dtype=np.int32)
    node_child1 = np.full(S, S, dtype=np.int32)
    node_child2 = np.full(S, S, dtype=np.int32)
    sub_start = np.empty(S, dtype=np.int32)
    sub_end = np.empty(S, dtype=np.int32)
    for node in range(S):
        s = post[node]
        if parent[node] >= 0:
            node_parent[s] = post[parent[node]]
        if left[node] >= 0:
            node_child1[s] = post[left[node]]
            node_child2[s] = post[right[node]]
        sub_start[s] = pre[node]
        sub_end[s] = pre[node] + size[node]
    # depth / ancestors-or-self count
    depth = np.zeros(S, dtype=np.int64)
    for s in range(S - 1, -1, -1):  # parents have larger postorder ids
        p = node_parent[s]
        if p >= 0:
            depth[s] = depth[p] + 1
    n_anc = depth + 1
    unnorm_row_max = -np.log2((S - n_anc).astype(np.float64))
    # compact levels: internal nodes grouped by depth, deepest first
    internal = np.nonzero(node_child1 < S)[0]
    levels = sorted(set(depth[internal].tolist()), reverse=True)
    lv_parents, lv_c1, lv_c2, ptr = [], [], [], [0]
    for d in levels:
        nodes = internal[depth[internal] == d]
        lv_parents.extend(nodes.tolist())
        lv_c1.extend(node_child1[nodes].tolist())
        lv_c2.extend(node_child2[nodes].tolist())
        ptr.append(len(lv_parents))
    leaves = np.nonzero(node_child1 >= S)[0]
    return {
        "S": S,
        "node_parent": node_parent,
        "node_child1": node_child1,
        "node_child2": node_child2,
        "node_subtree_start": sub_start,
        "node_subtree_end": sub_end,
        "max_ancestor_depth": int(n_anc.max()),
        "unnorm_row_max": unnorm_row_max.astype(np.float32),
        "compact_level_ptr": np.asarray(ptr, dtype=np.int64),
        "compact_level_parents": np.asarray(lv_parents, dtype=np.int32),
        "compact_level_child1": np.asarray(lv_c1, dtype=np.int32),
        "compact_level_child2": np.asarray(lv_c2, dtype=np.int32),
        "_species_leaves": leaves.astype(np.int64),
        "_depth": depth,
    }


# ----------------------------------------------------------------------------------------------
# gene topologies and the clade union
# ----------------------------------------------------------------------------------------------

def _nni(left, right, parent, root, n_moves, rng):
    """Random nearest-neighbour interchanges, in place (Python lists): for a random internal node
    v with an internal parent u, swap one child of v with v's sibling.  The root is unchanged."""
    internal = [i for i, x in enumerate(left) if x >= 0]
    n_int = len(internal)
    integers, random = rng.integers, rng.random
    for _ in range(n_moves):
        v = internal[int(integers(n_int))]
        u = parent[v]
        if u < 0:
            continue
        lu = left[u]
        w = right[u] if lu == v else lu
        if random() < 0.5:
            b = left[v]
            left[v] = w
        else:
            b = right[v]
            right[v] = w
        if left[u] == w:
            left[u] = b
        else:
            right[u] = b
        parent[w] = v
        parent[b] = u
    return root


def _clades(left, right, root, weights):
    """Postorder clade hashes (Python lists in, ``weights`` the leaf hashes as ints). Returns
    list of (hash, size, hash_left, hash_right) per internal node."""
    n_nodes = len(left)
    h = [0] * n_nodes
    sz = [1] * n_nodes
    out = []
    append = out.append
    stack = [root]
    pop, push = stack.pop, stack.append
    while stack:
        node = pop()
        if node < 0:                      # second visit of an internal node (encoded ~node)
            node = ~node
            lc, rc = left[node], right[node]
            hx = (h[lc] + h[rc]) & MASK64
            h[node] = hx
            sx = sz[lc] + sz[rc]
            sz[node] = sx
            append((hx, sx, h[lc], h[rc]))
            continue
        lc = left[node]
        if lc < 0:
            h[node] = weights[node]
            continue
        push(~node)
        push(right[node])
        push(lc)
    return out


def sample_topologies(cfg: ProblemConfig, species: dict, seed: int) -> dict:
    """The gene side of one family: ``T`` topologies over ``G`` gene leaves (one random base
    topology plus ``T-1`` copies perturbed by ``spr_moves`` nearest-neighbour interchanges), the
    gene leaves' hashes (random odd 64-bit integers) and their species leaves.

    Returns int32 ``left`` / ``right`` [T, 2G-1] (gene leaves are nodes 0..G-1 with children -1;
    internal nodes G..2G-2), int32 ``root`` [T], uint64 ``leaf_hash`` [G], int64
    ``leaf_species`` [G].  This is the input of the static builders (:func:`family_from_topologies`
    on the host, ``kbench_b200.builder`` on the device)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    G, T = cfg.n_genes, cfg.n_topologies
    weights = rng.integers(0, 2 ** 63, size=G, dtype=np.int64).astype(np.uint64) * _U64(2) + _U64(1)
    leaf_species = species["_species_leaves"][rng.integers(0, len(species["_species_leaves"]), size=G)]
    base_l, base_r, base_p, base_root = _random_merge_tree(G, rng)
    base_l, base_r, base_p = base_l.tolist(), base_r.tolist(), base_p.tolist()
    n_nodes = 2 * G - 1
    lefts = np.empty((T, n_nodes), dtype=np.int32)
    rights = np.empty((T, n_nodes), dtype=np.int32)
    roots = np.empty(T, dtype=np.int32)
    for t in range(T):
        left, right, parent = list(base_l), list(base_r), list(base_p)
        root = base_root
        if t > 0:
            root = _nni(left, right, parent, root, cfg.spr_moves, rng)
        lefts[t] = left
        rights[t] = right
        roots[t] = root
    return {"left": lefts, "right": rights, "root": roots, "leaf_hash": weights,
            "leaf_species": leaf_species.astype(np.int64)}


def make_family(cfg: ProblemConfig, species: dict, seed: int, *, alpha: float = 0.5,
                amalg_rounds: int = 2) -> dict:
    """One gene family: rows (clades) and their splits, in gene-clade hash space."""
    return family_from_topologies(sample_topologies(cfg, species, seed), alpha=alpha, amalg_rounds=amalg_rounds)


def family_from_topologies(topo: dict, *, alpha: float = 0.5, amalg_rounds: int = 2) -> dict:
    """Clade amalgamation of one family on the host: the union of the topologies' clades (rows)
    with their observed splits, widened by ``amalg_rounds`` rounds of splits one rearrangement
    away whose two parts are both clades, and log2 smoothed conditional split frequencies
    ``log2((count + alpha) / (n_obs + alpha * n_splits))`` per clade."""
    wlist = [int(w) for w in topo["leaf_hash"]]
    clade_size = {}
    clade_count = {}
    splits = {}        # clade hash -> {split key: observed count}
    for t in range(topo["left"].shape[0]):
        left, right = topo["left"][t].tolist(), topo["right"][t].tolist()
        for hx, sx, ha, hb in _clades(left, right, int(topo["root"][t]), wlist):
            clade_size[hx] = sx
            clade_count[hx] = clade_count.get(hx, 0) + 1
            key = (ha, hb) if ha < hb else (hb, ha)
            d = splits.setdefault(hx, {})
            d[key] = d.get(key, 0) + 1
    root_hash = sum(wlist) & MASK64
    leaf_hashes = wlist
    for g, hw in enumerate(leaf_hashes):
        clade_size[hw] = 1
    # amalgamation: splits a few rearrangements away whose parts are both clades
    cs_get = clade_size.get
    sp_get = splits.get
    for _round in range(amalg_rounds):
        added = {}
        for hx, d in splits.items():
            extra = {}
            for (ha, hb) in list(d):
                for (hc, ho) in ((ha, hb), (hb, ha)):
                    sub = sp_get(hc)
                    if not sub:
                        continue
                    s_ho = clade_size[ho]
                    for (h1, h2) in sub:
                        hy = (h2 + ho) & MASK64     # move h2 next to ho, keep h1
                        if cs_get(hy, 0) == clade_size[h2] + s_ho:
                            key = (h1, hy) if h1 < hy else (hy, h1)
                            if key not in d:
                                extra[key] = 0
                        hy = (h1 + ho) & MASK64     # move h1 next to ho, keep h2
                        if cs_get(hy, 0) == clade_size[h1] + s_ho:
                            key = (h2, hy) if h2 < hy else (hy, h2)
                            if key not in d:
                                extra[key] = 0
            if extra:
                added[hx] = extra
        if not added:
            break
        for hx, extra in added.items():
            splits[hx].update(extra)
    # log2 smoothed conditional split frequencies
    split_logp = {}
    for hx, d in splits.items():
        n_obs = sum(d.values())
        k = len(d)
        denom = n_obs + alpha * k
        split_logp[hx] = {key: math.log2((c + alpha) / denom) for key, c in d.items()}
    return {
        "clade_size": clade_size,
        "splits": split_logp,
        "leaf_hashes": leaf_hashes,
        "leaf_species": np.asarray(topo["leaf_species"], dtype=np.int64),
        "root_hash": root_hash,
    }


# ----------------------------------------------------------------------------------------------
# static layout
# ----------------------------------------------------------------------------------------------

def assemble_static(families: list[dict], species: dict) -> tuple[dict, dict]:
    """Merge families into one row space with waves by clade size. Returns (static, stats)."""
    S = species["S"]
    # rows grouped by (size, family); within a size, single-split parents first
    by_size: dict[int, list] = {}
    for f, fam in enumerate(families):
        for hx, sx in fam["clade_size"].items():
            by_size.setdefault(sx, []).append((f, hx))
    row_of = {}
    rows = []  # (family, hash)
    waves = []
    leaf_pos = [{hw: g for g, hw in enumerate(fam["leaf_hashes"])} for fam in families]
    for sx in sorted(by_size):
        members = by_size[sx]
        if sx == 1:
            members.sort(key=lambda fh: (fh[0], leaf_pos[fh[0]][fh[1]]))
        else:
            members.sort(key=lambda fh: (len(families[fh[0]]["splits"][fh[1]]) > 1, fh[0], fh[1]))
        start = len(rows)
        for fh in members:
            row_of[fh] = len(rows)
            rows.append(fh)
        waves.append((sx, start, len(members)))
    C = len(rows)
    leaf_state = np.full(C, -1, dtype=np.int32)
    item_idx = np.zeros(C, dtype=np.int64)
    for r, (f, hx) in enumerate(rows):
        item_idx[r] = f
    for f, fam in enumerate(families):
        for g, hw in enumerate(fam["leaf_hashes"]):
            leaf_state[row_of[(f, hw)]] = int(fam["leaf_species"][g])
    root_ids = np.asarray([row_of[(f, fam["root_hash"])] for f, fam in enumerate(families)],
                          dtype=np.int64)
    wave_metas = []
    n_split_total = 0
    max_w = 0
    k_children = 0
    for sx, start, W in waves:
        max_w = max(max_w, W)
        meta = {"start": start, "W": W}
        if sx == 1:
            wave_metas.append(meta)
            continue
        sl, sr, red, lsp = [], [], [], []
        eq1_count = 0
        ge2_ptr = [0]
        ge2_parents = []
        for local in range(W):
            f, hx = rows[start + local]
            d = families[f]["splits"][hx]
            items = sorted(d.items())
            for (ha, hb), lp in items:
                sl.append(row_of[(f, ha)])
                sr.append(row_of[(f, hb)])
                red.append(local)
                lsp.append(lp)
            if len(items) == 1:
                eq1_count += 1
            else:
                ge2_ptr.append(ge2_ptr[-1] + len(items))
                ge2_parents.append(local)
        n_eq1 = eq1_count
        meta.update({
            "sl": np.asarray(sl, dtype=np.int64),
            "sr": np.asarray(sr, dtype=np.int64),
            "reduce_idx": np.asarray(red, dtype=np.int64),
            "log_split_probs": np.asarray(lsp, dtype=np.float32),
            "n_eq1": n_eq1,
            "eq1_reduce_idx": np.asarray(red[:n_eq1], dtype=np.int64),
            "ge2_ptr": np.asarray(ge2_ptr, dtype=np.int64),
            "ge2_parent_ids": np.asarray(ge2_parents, dtype=np.int64),
            "ge2_max_fanout": int(max(np.diff(ge2_ptr))) if len(ge2_ptr) > 1 else 0,
        })
        n_split_total += len(sl)
        k_children += len(set(sl) | set(sr))
        wave_metas.append(meta)
    state_helpers = {k: v for k, v in species.items() if not k.startswith("_")}
    static = {
        "wave_layout": {
            "leaf_state_index": leaf_state,
            "root_row_ids": root_ids,
            "item_idx": item_idx,
            "wave_metas": wave_metas,
        },
        "state_helpers": state_helpers,
        "rate_item_idx": np.zeros(C, dtype=np.int64),
        "itemwise": False,
        "statewise": True,
    }
    n_internal = C - sum(len(f["leaf_hashes"]) for f in families)
    stats = {
        "C": C,
        "n_waves": len(wave_metas),
        "max_W": max_w,
        "n_splits": n_split_total,
        "splits_per_internal_row": n_split_total / max(1, n_internal),
        "K_children": k_children,
    }
    return static, stats


def make_theta(S: int, seed: int) -> np.ndarray:
    """theta[S,3] = log2 of per-column rates drawn as exp(N(ln 0.05, 0.5^2)).

    Column order follows the reference parameterisation (``extract_parameters.py:25-34``):
    theta[:,0] -> duplication, theta[:,1] -> loss, theta[:,2] -> transfer, each a log2-odds
    against speciation.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    ln_rate = rng.normal(math.log(0.05), 0.5, size=(S, 3))
    return (ln_rate / math.log(2.0)).astype(np.float32)


def generate(config: int | ProblemConfig, *, seed: int | None = None, n_families: int | None = None,
             family_offset: int = 0, as_torch: bool = True, solver_options: dict | None = None):
    """Build a ``captured`` dict: ``{"meta", "static", "inputs"}``.

    ``seed`` defaults to ``1000 * config``; family ``f`` uses seed ``seed + 1 + f``; the species
    tree uses ``seed`` and theta ``seed + 7``. ``n_families``/``family_offset`` select a slice of a
    batched config (each rank of a sharded run builds only its own families).
    """
    cfg = CONFIGS[config] if isinstance(config, int) else config
    cfg_id = config if isinstance(config, int) else 0
    seed = 1000 * cfg_id if seed is None else int(seed)
    nf = cfg.n_families if n_families is None else int(n_families)
    species = make_species_tree(cfg.n_species, seed)
    fams = [make_family(cfg, species, seed + 1 + family_offset + f) for f in range(nf)]
    static, stats = assemble_static(fams, species)
    S = species["S"]
    theta = make_theta(S, seed + 7)
    so = dict(cfg.solver_options)
    if solver_options:
        so.update(solver_options)
    meta = {
        "label": cfg.name, "config": cfg_id, "seed": seed, "S": S, "C": stats["C"],
        "n_items": nf, "family_offset": family_offset, "solver_options": so,
        "theta_columns": ["log2_dup", "log2_loss", "log2_transfer"], **stats,
    }
    captured = {
        "meta": meta,
        "static": static,
        "inputs": {"theta": theta, "col_weights": np.zeros(S, dtype=np.float32)},
    }
    return to_torch(captured) if as_torch else captured


def to_torch(obj):
    """Recursively convert numpy arrays to torch tensors (CPU)."""
    import torch
    if isinstance(obj, np.ndarray):
        if obj.size == 0:
            # torch.from_numpy gives empty arrays a zero stride, which byte views (the reference
            # capture's content hash) reject; an ordinary empty tensor has unit strides
            return torch.empty(obj.shape, dtype=torch.from_numpy(np.zeros(1, obj.dtype)).dtype)
        return torch.from_numpy(np.ascontiguousarray(obj))
    if isinstance(obj, dict):
        return {k: to_torch(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [to_torch(v) for v in obj]
    return obj
