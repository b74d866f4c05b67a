"""Device-side species-tree tables shared by the kernels.

``tables(node_parent, ...)`` returns (and caches, keyed by the ``node_parent`` storage like the
reference's own host caches, ``kbench/core/kernels/wave_step.py:35-55``) the pointer-doubling
ancestor table used for the ancestor-or-self path sums and int32/int64 copies of the compact
level arrays used for bottom-up subtree sums.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class TreeTables:
    S: int
    K: int
    jumps: torch.Tensor          # [max(K,1), S] int32
    parent: torch.Tensor         # [S] int32
    child1: torch.Tensor         # [S] int32
    child2: torch.Tensor         # [S] int32
    lv_ptr: torch.Tensor | None  # [L+1] int64
    lv_par: torch.Tensor | None
    lv_c1: torch.Tensor | None
    lv_c2: torch.Tensor | None
    n_levels: int
    packed: torch.Tensor | None = None  # [4,S] uint32 per-column tables, see pack_columns()


_CACHE: dict = {}
NONE16 = 0xFFFF


def engine_width(S: int) -> tuple[int, int]:
    """(threads per CTA, columns per thread) of the engine kernels; their product is the padded row
    width NTV >= S + 1 (S is odd for a binary tree, NTV is even)."""
    bd = 1024 if S > 1024 else max(32, ((S + 31) // 32) * 32)
    v = (S + bd - 1) // bd
    vpt = 1 if v <= 1 else 2 if v <= 2 else 4 if v <= 4 else 8
    if bd * vpt < S + 1:  # keep a zero padding column
        vpt *= 2
    return bd, vpt


def tour_layout(S: int):
    """(NTV, threads, columns per thread) of the forward tour kernel, or None where it does not
    apply (rows wider than 4096 padded columns): NTV is the smallest power of two > S (at least
    64), 8 columns per thread where the row is wide enough.  Mirrors ``tour_layout`` in
    csrc/kb_engine.cu."""
    ntv = max(64, 1 << int(S).bit_length())
    if ntv > 4096:
        return None
    vf = min(8, ntv // 32)
    return ntv, ntv // vf, vf


def tour_phys(i, vf: int):
    """Swizzled shared-memory position of logical tour index i in the forward tour kernel: thread
    t scans the 2*vf entries [t*2vf, (t+1)*2vf) as vf/2 float4 groups whose order inside the chunk
    is XOR-permuted by (t // (8 // groups)) so a quarter-warp's vector loads hit distinct banks."""
    import numpy as np
    i = np.asarray(i, dtype=np.int64)
    ch = 2 * vf
    q_n = ch // 4
    if q_n == 1:
        return i
    t, j = i // ch, i % ch
    q, r = j // 4, j % 4
    sw = (t // (8 // q_n)) & (q_n - 1)
    return t * ch + 4 * (q ^ sw) + r


def pack_forward(parent, child1, child2, sub_start, sub_end):
    """[3, NTV] uint32 tables (viewed as int32) of the forward tour kernel, for NTV, VF =
    tour_layout(S):

    row 0  children columns c1 | c2 << 16 (a missing child -> the zero column Z = NTV-1)
    row 1  BYTE offsets of the children's enter slots in a tour buffer (lo | hi << 16)
    row 2  BYTE offsets of the column's own enter | exit slots
    """
    import numpy as np
    S = len(parent)
    lay = tour_layout(S)
    if lay is None:
        raise ValueError("row too wide for the forward tour kernel")
    ntv, _, vf = lay
    pk = pack_columns(parent, child1, child2, sub_start, sub_end, ntv=ntv).view(np.uint32).astype(np.int64)
    c1, c2 = pk[0] & 0xFFFF, pk[0] >> 16
    enter, exit_ = pk[1] & 0xFFFF, pk[1] >> 16
    be, bx = 4 * tour_phys(enter, vf), 4 * tour_phys(exit_, vf)
    if max(be.max(), bx.max()) > 0xFFFF:
        raise ValueError("tour byte offsets exceed 16 bits")
    out = np.stack([c1 | (c2 << 16), be[c1] | (be[c2] << 16), be | (bx << 16)])
    return out.astype(np.uint32).view(np.int32)


def tour_phys_pair(i, vf: int):
    """Swizzled position (in float2 entries) of logical tour index i in the two-direction tour layout
    of the tangent kernel: thread t scans the 2*vf entries [t*2vf, (t+1)*2vf) as vf float4 groups
    (two entries each) whose order inside the chunk is XOR-permuted by (t // (8 // vf))."""
    import numpy as np
    i = np.asarray(i, dtype=np.int64)
    ch = 2 * vf
    t, j = i // ch, i % ch
    q, r = j // 2, j % 2
    sw = 0 if vf == 1 else (t // (8 // vf)) & (vf - 1)
    return t * ch + 2 * (q ^ sw) + r


def pack_tour_pair(parent, child1, child2, sub_start, sub_end):
    """[NTV] uint32 (viewed as int32): byte offsets of each column's enter | exit << 16 slots in
    the two-direction (float2) tour layout, for NTV, VF = tour_layout(S)."""
    import numpy as np
    S = len(parent)
    lay = tour_layout(S)
    if lay is None:
        raise ValueError("row too wide for the tour kernels")
    ntv, _, vf = lay
    pk = pack_columns(parent, child1, child2, sub_start, sub_end, ntv=ntv).view(np.uint32).astype(np.int64)
    be = 8 * tour_phys_pair(pk[1] & 0xFFFF, vf)
    bx = 8 * tour_phys_pair(pk[1] >> 16, vf)
    if max(be.max(), bx.max()) > 0xFFFF:
        raise ValueError("pair tour byte offsets exceed 16 bits")
    return (be | (bx << 16)).astype(np.uint32).view(np.int32)


def pack_columns(parent, child1, child2, sub_start, sub_end, ntv=None):
    """Per-column 32-bit tables (two 16-bit fields each) read once per CTA by the engine kernels:

    row 0  children:   c1 | c2 << 16            (0xFFFF = no child)
    row 1  Euler tour: enter | exit << 16        positions in the 2S-long tour (+P at enter,
                                                 -P at exit), so the inclusive prefix at enter(x)
                                                 is the ancestor-or-self path sum of x
    row 2  preorder:   pre | pre_end << 16       subtree of x = preorder range [pre, pre_end)
    row 3  parent:     parent | (x is the parent's first child) << 16   (0xFFFF = root)

    With ``ntv`` (padded to ntv columns) a fifth row is indexed by PREORDER POSITION q instead of
    by column (the backward kernel's Neumann sweep runs with thread t owning positions
    [t*VPT, (t+1)*VPT)):

    row 4  position q: pre_end(x) | pre(parent(x)) << 16   for the column x with pre(x) = q
    """
    import numpy as np
    par = np.asarray(parent, dtype=np.int64)
    c1 = np.asarray(child1, dtype=np.int64)
    c2 = np.asarray(child2, dtype=np.int64)
    pre = np.asarray(sub_start, dtype=np.int64)
    pre_end = np.asarray(sub_end, dtype=np.int64)
    S = par.shape[0]
    if S >= NONE16:
        raise ValueError("packed column tables need S < 65535")
    depth = np.zeros(S, dtype=np.int64)
    order = np.argsort(pre)  # preorder: parents before children
    for x in order:
        p = par[x]
        if 0 <= p < S:
            depth[x] = depth[p] + 1
    size = pre_end - pre
    enter = 2 * pre - depth
    exit_ = 2 * (pre + size) - depth - 1
    v1 = np.where((c1 >= 0) & (c1 < S), c1, NONE16)
    v2 = np.where((c2 >= 0) & (c2 < S), c2, NONE16)
    pv = np.where((par >= 0) & (par < S), par, NONE16)
    first = np.zeros(S, dtype=np.int64)
    ok = pv != NONE16
    first[ok] = (c1[par[ok]] == np.nonzero(ok)[0]).astype(np.int64)
    out = np.stack([v1 | (v2 << 16), enter | (exit_ << 16), pre | (pre_end << 16), pv | (first << 16)])
    if ntv is not None:
        # padded columns S..ntv-1 (always zero in the kernels): children/parent point at the zero
        # column Z = ntv-1, tour slots 2S.. and preorder slots S.. are their own
        Z = ntv - 1
        pad = np.arange(S, ntv, dtype=np.int64)
        ext = np.stack([Z | (Z << 16) + 0 * pad,
                        (2 * pad) | ((2 * pad + 1) << 16),
                        pad | (pad << 16),
                        Z + 0 * pad])
        real = out.copy()
        # real columns: invalid child / parent -> Z
        c1f = np.where(v1 == NONE16, Z, v1)
        c2f = np.where(v2 == NONE16, Z, v2)
        pf = np.where(pv == NONE16, Z, pv)
        real[0] = c1f | (c2f << 16)
        real[3] = pf | (first << 16)
        out = np.concatenate([real, ext], axis=1)
        pre_p = out[2] & 0xFFFF
        end_p = out[2] >> 16
        par_p = out[3] & 0xFFFF
        col_of = np.empty(ntv, dtype=np.int64)
        col_of[pre_p] = np.arange(ntv, dtype=np.int64)  # preorder (padded) is a permutation
        pos_row = end_p[col_of] | (pre_p[par_p[col_of]] << 16)
        out = np.concatenate([out, pos_row[None, :]], axis=0)
    return out.astype(np.uint32).view(np.int32)


_CACHE: dict = {}


def rounds_for_depth(max_ancestor_depth: int) -> int:
    """Doubling rounds so that 2^K >= the longest root path (nodes, counting self)."""
    d = max(1, int(max_ancestor_depth))
    return 0 if d <= 1 else int(math.ceil(math.log2(d)))


def _i32(t, device):
    return t.to(device=device, dtype=torch.int32).contiguous()


def tables(node_parent, node_child1, node_child2, max_ancestor_depth, *, compact_level_ptr=None,
           compact_level_parents=None, compact_level_child1=None, compact_level_child2=None) -> TreeTables:
    device = node_parent.device
    S = int(node_parent.numel())
    key = (node_parent.data_ptr(), node_child1.data_ptr(), S, int(max_ancestor_depth),
           None if compact_level_ptr is None else compact_level_ptr.data_ptr(), device.index)
    hit = _CACHE.get(key)
    if hit is not None:
        return hit
    parent = _i32(node_parent, device)
    c1 = _i32(node_child1, device)
    c2 = _i32(node_child2, device)
    K = rounds_for_depth(max_ancestor_depth)
    jumps = torch.empty((max(K, 1), S), dtype=torch.int32, device=device)
    if K:
        _lib.call("kb_build_jumps", parent.data_ptr(), S, K, jumps.data_ptr(), _lib.stream_handle(device))
    if compact_level_ptr is None:
        compact_level_ptr, compact_level_parents, compact_level_child1, compact_level_child2 = \
            derive_levels(node_parent, node_child1, node_child2)
    if compact_level_ptr is not None:
        lv_ptr = compact_level_ptr.to(device=device, dtype=torch.int64).contiguous()
        lv_par = _i32(compact_level_parents, device)
        lv_c1 = _i32(compact_level_child1, device)
        lv_c2 = _i32(compact_level_child2, device)
        n_levels = int(lv_ptr.numel()) - 1
    else:
        lv_ptr = lv_par = lv_c1 = lv_c2 = None
        n_levels = 0
    tt = TreeTables(S, K, jumps, parent, c1, c2, lv_ptr, lv_par, lv_c1, lv_c2, n_levels)
    # keep the source tensors alive with the entry so their addresses are not reused
    _CACHE[key] = tt
    tt._keep = (node_parent, node_child1, node_child2, compact_level_ptr)  # type: ignore[attr-defined]
    return tt


def children_from_parent(node_parent):
    """(node_child1, node_child2) of a binary tree given by its parent array: the smaller and the
    larger child index of each internal node, ``S`` (no child) for leaves."""
    par = node_parent.detach().to("cpu", torch.int64)
    S = int(par.numel())
    c1 = torch.full((S,), S, dtype=torch.int64)
    c2 = torch.full((S,), S, dtype=torch.int64)
    for s in range(S):
        p = int(par[s])
        if 0 <= p < S:
            if int(c1[p]) == S:
                c1[p] = s
            else:
                c2[p] = s
    return c1.to(node_parent.device), c2.to(node_parent.device)


def derive_levels(node_parent, node_child1, node_child2):
    """Compact levels (internal nodes grouped by depth, deepest level first) from the parent
    and child arrays, for callers that did not pass the precomputed ones."""
    par = node_parent.detach().to("cpu", torch.int64)
    c1 = node_child1.detach().to("cpu", torch.int64)
    c2 = node_child2.detach().to("cpu", torch.int64)
    S = int(par.numel())
    depth = [0] * S
    # depth by walking up (trees here are shallow); memoised
    for s in range(S):
        d, cur = 0, int(par[s])
        while 0 <= cur < S:
            d += 1
            cur = int(par[cur])
        depth[s] = d
    internal = [s for s in range(S) if 0 <= int(c1[s]) < S]
    levels = sorted({depth[s] for s in internal}, reverse=True)
    ptr, lp, l1, l2 = [0], [], [], []
    for d in levels:
        nodes = [s for s in internal if depth[s] == d]
        lp += nodes
        l1 += [int(c1[s]) for s in nodes]
        l2 += [int(c2[s]) for s in nodes]
        ptr.append(len(lp))
    dev = node_parent.device
    return (torch.tensor(ptr, dtype=torch.int64, device=dev), torch.tensor(lp, dtype=torch.int32, device=dev),
            torch.tensor(l1, dtype=torch.int32, device=dev), torch.tensor(l2, dtype=torch.int32, device=dev))


def from_helpers(sh: dict) -> TreeTables:
    tt = tables(sh["node_parent"], sh["node_child1"], sh["node_child2"], int(sh["max_ancestor_depth"]),
                compact_level_ptr=sh.get("compact_level_ptr"),
                compact_level_parents=sh.get("compact_level_parents"),
                compact_level_child1=sh.get("compact_level_child1"),
                compact_level_child2=sh.get("compact_level_child2"))
    if tt.packed is None:
        arrs = [sh[k].detach().cpu().numpy() for k in ("node_parent", "node_child1", "node_child2",
                                                        "node_subtree_start", "node_subtree_end")]
        dev = sh["node_parent"].device
        tt.packed = torch.from_numpy(pack_columns(*arrs)).to(dev).contiguous()
        bd, vpt = engine_width(int(sh["S"]))
        tt.packed_pad = torch.from_numpy(pack_columns(*arrs, ntv=bd * vpt)).to(dev).contiguous()
        tt.tour = (torch.from_numpy(pack_forward(*arrs)).to(dev).contiguous()
                   if tour_layout(int(sh["S"])) is not None else None)
        tt.tour_pair = (torch.from_numpy(pack_tour_pair(*arrs)).to(dev).contiguous()
                        if tour_layout(int(sh["S"])) is not None else None)
    return tt
