"""The fused B200 engine (default driver of ``runtime.run_forward`` / ``run_backward``).

Schedule.  The reference processes rows in "waves" of equal clade size, smallest first, and calls
``pi_iters`` wave-step launches per wave plus a split-reduction launch (``kbench/core/inference/
forward.py:60-115``).  A row only depends on the final Pi/Pibar of its split children, so any
topological banding gives bit-identical per-row arithmetic.  The engine re-bands the rows into
dependency levels (level 0: leaf rows; otherwise 1 + the deepest child level) once per problem:
at the large config that is 186 levels instead of 1,666 size-waves, and each level is ONE launch
(``kb_level_forward``) that does the split reduction and all iterations of every row of the level.
The backward runs the levels in reverse with one launch each (``kb_level_backward``).

The engine supports the layouts of every benchmark config (one shared item row: ``statewise`` and
not ``itemwise``); anything else is routed to the reference-structured driver of ``glue.py``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, glue, tree
from .kernels._common import f32, i32, i64


@dataclass
class LevelPlan:
    n_levels: int
    level_ptr: list            # row offsets of each level in ``rows`` (host ints)
    rows: torch.Tensor         # int32 [C] rows in level order
    split_ptr: torch.Tensor    # int64 [C+1] CSR of each listed row's splits
    sl: torch.Tensor           # int64 [N]
    sr: torch.Tensor
    lsp: torch.Tensor          # f32 [N]
    level_of: np.ndarray       # level of every row (host; None for a plan built on the device)
    children_per_level: list   # distinct child rows referenced per level (for the traffic model)
    n_splits: int
    # dataflow schedule (one persistent launch): splits in row-id order, dependency counts, parents
    row_split_ptr: torch.Tensor  # int64 [C+1]
    sl_r: torch.Tensor           # int64 [N]
    sr_r: torch.Tensor
    lsp_r: torch.Tensor          # f32 [N]
    dep0: torch.Tensor           # int32 [C] distinct child rows
    ready0: torch.Tensor         # int32 rows with dep0 == 0
    par_ptr: torch.Tensor        # int64 [C+1] distinct parent rows of each row
    par_idx: torch.Tensor        # int32
    dep_b: torch.Tensor          # int32 [C] distinct parent rows (backward dependencies)
    ready_b: torch.Tensor        # int32 rows without parents
    child_ptr: torch.Tensor      # int64 [C+1] distinct child rows of each row
    child_idx: torch.Tensor      # int32


def _sorted_unique(keys: np.ndarray) -> np.ndarray:
    """Distinct values of an int64 array, ascending (a sort and one comparison pass)."""
    k = np.sort(keys)
    return k[np.concatenate(([True], k[1:] != k[:-1]))] if k.shape[0] else k


def build_plan(static) -> LevelPlan:
    """Dependency levels and the per-row split CSR, from the reference wave layout (on the device
    by ``kb_plan_build`` when the static carries the flat split arrays of a device-built layout,
    else on the host)."""
    cached = getattr(static, "_plan", None)
    if cached is not None:
        return cached
    flat = getattr(static, "flat_layout", None)
    if flat is not None and flat["sl"].is_cuda:
        static._plan = build_plan_device(static)
        return static._plan
    wl = static.wave_layout
    dev = wl["leaf_state_index"].device
    C = int(wl["leaf_state_index"].numel())
    level = np.zeros(C, dtype=np.int64)
    par, sls, srs, lsps = [], [], [], []
    for meta in wl["wave_metas"]:
        if "sl" not in meta:
            continue
        ws = int(meta["start"])
        sl = meta["sl"].detach().cpu().numpy().astype(np.int64)
        sr = meta["sr"].detach().cpu().numpy().astype(np.int64)
        p = ws + meta["reduce_idx"].detach().cpu().numpy().astype(np.int64)
        n = sl.shape[0]
        lp = meta.get("log_split_probs")
        lp = np.zeros(n, np.float32) if lp is None else lp.detach().cpu().numpy().reshape(n).astype(np.float32)
        np.maximum.at(level, p, np.maximum(level[sl], level[sr]) + 1)
        par.append(p); sls.append(sl); srs.append(sr); lsps.append(lp)
    if par:
        par = np.concatenate(par); sls = np.concatenate(sls); srs = np.concatenate(srs)
        lsps = np.concatenate(lsps)
    else:
        par = sls = srs = np.zeros(0, np.int64)
        lsps = np.zeros(0, np.float32)
    # stable argsorts and unique over int64 keys (row * C + row) keep this linear-ish for the
    # multi-million-row statics of family batches
    order_rows = np.argsort(level, kind="stable")
    pos = np.empty(C, dtype=np.int64)
    pos[order_rows] = np.arange(C)
    order_splits = np.argsort(pos[par], kind="stable")
    counts = np.bincount(pos[par], minlength=C) if par.shape[0] else np.zeros(C, np.int64)
    split_ptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    n_levels = int(level.max()) + 1 if C else 0
    level_ptr = [0] + np.cumsum(np.bincount(level, minlength=n_levels)).tolist()
    sp_sorted = par[order_splits]
    lv_of_split = level[sp_sorted]
    s_l, s_r = sls[order_splits], srs[order_splits]
    if par.shape[0]:  # distinct child rows per level: unique (level, child) keys
        lk = _sorted_unique(np.concatenate([lv_of_split * C + s_l, lv_of_split * C + s_r]))
        children = np.bincount(lk // C, minlength=n_levels).tolist()
    else:
        children = [0] * n_levels
    # dataflow arrays
    order_r = np.argsort(par, kind="stable") if par.shape[0] else np.zeros(0, np.int64)
    cnt_r = np.bincount(par, minlength=C) if par.shape[0] else np.zeros(C, np.int64)
    row_split_ptr = np.concatenate([[0], np.cumsum(cnt_r)]).astype(np.int64)
    if par.shape[0]:
        pk = _sorted_unique(np.concatenate([par * C + sls, par * C + srs]))  # sorted by (parent, child)
        pairs = np.stack([pk // C, pk % C], axis=1)
    else:
        pairs = np.zeros((0, 2), np.int64)
    dep0 = np.bincount(pairs[:, 0], minlength=C).astype(np.int32) if pairs.shape[0] else np.zeros(C, np.int32)
    by_child = pairs[np.argsort(pairs[:, 1] * C + pairs[:, 0])] if pairs.shape[0] else pairs
    cnt_c = np.bincount(by_child[:, 1], minlength=C) if pairs.shape[0] else np.zeros(C, np.int64)
    par_ptr = np.concatenate([[0], np.cumsum(cnt_c)]).astype(np.int64)
    ready0 = np.nonzero(dep0 == 0)[0].astype(np.int32)
    dep_b = cnt_c.astype(np.int32)
    ready_b = np.nonzero(dep_b == 0)[0].astype(np.int32)
    cnt_p = np.bincount(pairs[:, 0], minlength=C) if pairs.shape[0] else np.zeros(C, np.int64)
    child_ptr = np.concatenate([[0], np.cumsum(cnt_p)]).astype(np.int64)  # pairs are sorted by parent
    plan = LevelPlan(
        n_levels=n_levels, level_ptr=level_ptr,
        rows=torch.from_numpy(order_rows.astype(np.int32)).to(dev),
        split_ptr=torch.from_numpy(split_ptr).to(dev),
        sl=torch.from_numpy(s_l.astype(np.int64)).to(dev),
        sr=torch.from_numpy(s_r.astype(np.int64)).to(dev),
        lsp=torch.from_numpy(lsps[order_splits].astype(np.float32)).to(dev),
        level_of=level, children_per_level=children, n_splits=int(par.shape[0]),
        row_split_ptr=torch.from_numpy(row_split_ptr).to(dev),
        sl_r=torch.from_numpy(sls[order_r].astype(np.int64)).to(dev),
        sr_r=torch.from_numpy(srs[order_r].astype(np.int64)).to(dev),
        lsp_r=torch.from_numpy(lsps[order_r].astype(np.float32)).to(dev),
        dep0=torch.from_numpy(dep0).to(dev), ready0=torch.from_numpy(ready0).to(dev),
        par_ptr=torch.from_numpy(par_ptr).to(dev),
        par_idx=torch.from_numpy(by_child[:, 0].astype(np.int32)).to(dev),
        dep_b=torch.from_numpy(dep_b).to(dev), ready_b=torch.from_numpy(ready_b).to(dev),
        child_ptr=torch.from_numpy(child_ptr).to(dev),
        child_idx=torch.from_numpy(pairs[:, 1].astype(np.int32)).to(dev),
    )
    static._plan = plan
    return plan


def build_plan_device(static) -> LevelPlan:
    """:func:`build_plan` on the device from ``static.flat_layout`` (the row-ordered split arrays a
    device-built layout carries): the same arrays, computed by ``kb_plan_build``."""
    fl = static.flat_layout
    dev = fl["sl"].device
    C = int(static.wave_layout["leaf_state_index"].numel())
    N = int(fl["sl"].numel())
    wsp = np.asarray(fl["wave_split_ptr"], dtype=np.int64)
    nw = int(wsp.shape[0]) - 1
    nbytes = np.zeros(1, dtype=np.int64)
    _lib.call("kb_plan_workspace", C, N, nbytes.ctypes.data)
    ws = torch.empty(int(nbytes[0]), dtype=torch.uint8, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    i64 = dict(dtype=torch.int64, device=dev)
    rows, split_ptr = torch.empty(C, **i32), torch.empty(C + 1, **i64)
    sl_lv, sr_lv = torch.empty(N, **i64), torch.empty(N, **i64)
    lsp_lv = torch.empty(N, dtype=torch.float32, device=dev)
    dep0, ready0, dep_b, ready_b = (torch.empty(C, **i32) for _ in range(4))
    par_ptr, child_ptr = torch.empty(C + 1, **i64), torch.empty(C + 1, **i64)
    par_idx, child_idx = torch.empty(max(2 * N, 1), **i32), torch.empty(max(2 * N, 1), **i32)
    level_ptr = np.zeros(nw + 1, dtype=np.int64)
    children = np.zeros(nw, dtype=np.int64)
    sizes = np.zeros(5, dtype=np.int64)
    p = _lib.ptr
    _lib.call("kb_plan_build", C, N, nw, wsp.ctypes.data, p(fl["split_row"]), p(fl["sl"]), p(fl["sr"]),
              p(fl["lsp"]), p(fl["row_split_ptr"]), p(ws), int(nbytes[0]), p(rows), p(split_ptr), p(sl_lv), p(sr_lv),
              p(lsp_lv), p(dep0), p(ready0), p(par_ptr), p(par_idx), p(dep_b), p(ready_b), p(child_ptr),
              p(child_idx), level_ptr.ctypes.data, children.ctypes.data, sizes.ctypes.data,
              _lib.stream_handle(dev))
    n_levels, P, n_r0, n_rb = (int(x) for x in sizes[:4])
    if int(sizes[4]):
        raise RuntimeError(f"kb_plan_build: status {int(sizes[4])}")
    del ws
    return LevelPlan(
        n_levels=n_levels, level_ptr=level_ptr[:n_levels + 1].tolist(), rows=rows, split_ptr=split_ptr,
        sl=sl_lv, sr=sr_lv, lsp=lsp_lv, level_of=None, children_per_level=children[:n_levels].tolist(), n_splits=N,
        row_split_ptr=fl["row_split_ptr"], sl_r=fl["sl"], sr_r=fl["sr"], lsp_r=fl["lsp"],
        dep0=dep0, ready0=ready0[:n_r0], par_ptr=par_ptr, par_idx=par_idx[:P], dep_b=dep_b, ready_b=ready_b[:n_rb],
        child_ptr=child_ptr, child_idx=child_idx[:P],
    )


# Relative cost of one split against the rest of a row (measured on config 3: forward ~5.3k of
# ~80k SM cycles per row besides its splits; backward ~17k of ~100k).
FWD_SPLIT_COST = 0.066
BWD_SPLIT_COST = 0.17


def start_order(plan: LevelPlan, direction: str, n_workers: int) -> torch.Tensor:
    """A fixed start order for a dataflow pass (int32 [C], device): the order in which rows START
    in a critical-path list schedule of the pass on ``n_workers`` CTAs (``kb_list_schedule``, host
    code), with a row's cost 1 + (FWD|BWD)_SPLIT_COST x its splits.  Every row comes after the rows
    it waits for -- its children in the forward, its parents in the backward -- and the rows of the
    longest remaining chains start first, which shortens the pass's tail (forward) or ramp
    (backward) where few rows are ready.  Cached on the plan."""
    key = f"_order_{direction}_{n_workers}"
    cached = getattr(plan, key, None)
    if cached is not None:
        return cached
    rsp = plan.row_split_ptr.cpu().numpy()
    C = rsp.shape[0] - 1
    w = FWD_SPLIT_COST if direction == "forward" else BWD_SPLIT_COST
    cost = np.ascontiguousarray(1.0 + w * np.diff(rsp).astype(np.float64))
    cp, ci = plan.child_ptr.cpu().numpy(), plan.child_idx.cpu().numpy()
    pp, pi = plan.par_ptr.cpu().numpy(), plan.par_idx.cpu().numpy()
    (pred_ptr, pred_idx), (succ_ptr, succ_idx) = ((cp, ci), (pp, pi)) if direction == "forward" else ((pp, pi), (cp, ci))
    arrs = [np.ascontiguousarray(a) for a in (pred_ptr.astype(np.int64), pred_idx.astype(np.int32),
                                              succ_ptr.astype(np.int64), succ_idx.astype(np.int32))]
    order = np.empty(C, dtype=np.int32)
    span = np.zeros(1, dtype=np.float64)
    _lib.call("kb_list_schedule", C, *(a.ctypes.data for a in arrs), cost.ctypes.data, int(n_workers),
              order.ctypes.data, span.ctypes.data)
    out = torch.from_numpy(order).to(plan.rows.device)
    setattr(plan, key, out)
    return out


def _one_family(static) -> bool:
    """Whether the static holds one family: its chains of dependent rows are what a pass's tail
    and ramp are made of, and the fixed start order pays; a batch of families keeps the SMs busy
    with independent chains in any order (and a multi-million-row schedule costs host time)."""
    return int(static.wave_layout["root_row_ids"].numel()) == 1


def _forward_ctas(S) -> int:
    """CTAs of the dataflow forward's persistent grid for S columns on the current device."""
    import ctypes
    n = ctypes.c_int(0)
    _lib.call("kb_forward_ctas", S, ctypes.byref(n))
    return int(n.value)


def supported(static) -> bool:
    """The fused engine's layouts: one shared item row (statewise, not itemwise) and rows of at
    most 4,095 columns (the tour kernels' 4,096-column padded width); anything else runs on the
    call-by-call driver of ``glue.py``."""
    S = int(static.state_helpers["S"])
    return bool(static.statewise) and not bool(static.itemwise) and tree.tour_layout(S) is not None


class _Topo:
    """Device arrays of the species tree the engine kernels take."""

    def __init__(self, sh):
        self.tt = tree.from_helpers(sh)
        self.pre = i32(sh["node_subtree_start"])
        self.pre_end = i32(sh["node_subtree_end"])


def _topo(static):
    t = getattr(static, "_topo", None)
    if t is None:
        t = _Topo(static.state_helpers)
        static._topo = t
    return t


class LevelTimer:
    """Optional per-level CUDA-event timing of the engine's level kernels (set
    ``static._level_timer = LevelTimer()``); events are recorded on the launching stream."""

    def __init__(self):
        self.events = {"kb_level_forward": [], "kb_level_backward": []}

    def wrap(self, name, level, fn):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        self.events.setdefault(name, []).append((level, a, b))

    def totals(self):
        """{kernel: (total_ms, n_launches, per-level list of (level, ms))} after a sync."""
        out = {}
        for name, evs in self.events.items():
            per = [(lv, a.elapsed_time(b)) for lv, a, b in evs]
            out[name] = (sum(t for _, t in per), len(per), per)
        return out

    def reset(self):
        for v in self.events.values():
            v.clear()


def _launch(static, name, level, *args):
    timer = getattr(static, "_level_timer", None)
    if timer is None:
        _lib.call(name, *args)
    else:
        timer.wrap(name, level, lambda: _lib.call(name, *args))


@dataclass
class Prep:
    """Everything the level kernels need that depends only on theta and the species tree (so it
    is shared by every chunk of a family batch): parameters, the E fixed point and the per-column
    constants of the row update."""
    pS: torch.Tensor
    pD: torch.Tensor
    pL: torch.Tensor
    mc: torch.Tensor
    clp: torch.Tensor
    ucw: bool
    E: torch.Tensor
    E_s1: torch.Tensor
    E_s2: torch.Tensor
    Ebar: torch.Tensor
    k: dict
    lin: torch.Tensor
    k4: torch.Tensor | None   # tour kernel constants [G, NTV, 4] (None where the tour kernel does not apply)
    # constants outside the linear iteration's exact range (every row in log space), as a device
    # int32 word: the dataflow forward reads it on the device, without a host round trip
    force_log_dev: torch.Tensor | None = None

    @property
    def force_log(self) -> bool:
        return self.force_log_dev is not None and bool(self.force_log_dev.item())


# Smallest log2 of a linear-iteration constant for which the forward kernels' linear-space update is
# exact: nonzero row values are kept >= 2^-100 of the row scale (smaller ones send the row to the
# log-space iteration), so a product with a constant >= 2^-26 stays >= 2^-126, a normal fp32 number.
LINEAR_MIN_LOG2 = -26.0


def linear_range_flag(k: dict) -> torch.Tensor:
    """Device int32 [1]: 1 unless every finite exponent of the forward's linear constants --
    log2(2^dl + 2^ebar) (at least max(dl, ebar)), mc + e, sl1, sl2 -- is at least
    ``LINEAR_MIN_LOG2``.  Below it (extreme rates) a term could underflow to zero where the
    reference's log-space update keeps it finite, so the engine then runs every row's iterations
    in log space."""
    ex = torch.stack([torch.maximum(k["dl"], k["ebar"]), k["mc"] + k["e"], k["sl1"], k["sl2"]])
    return ((ex < LINEAR_MIN_LOG2) & torch.isfinite(ex)).any().reshape(1).to(torch.int32)


def linear_range_ok(k: dict) -> bool:
    """Host view of :func:`linear_range_flag` (one synchronisation)."""
    return not bool(linear_range_flag(k).item())


@torch.no_grad()
def prepare(static, theta, col_weights) -> Prep:
    """Parameters, E fixed point (``glue.solve_parameters`` / ``glue.solve_e``) and the linear
    constants ``2^dl + 2^ebar, 2^(mc+e), 2^sl1, 2^sl2`` of the forward's row update."""
    S = int(static.state_helpers["S"])
    pS, pD, pL, mc, clp, ucw = glue.solve_parameters(static, theta, col_weights)
    E, E_s1, E_s2, Ebar = glue.solve_e(static, pS, pD, pL, mc, clp, ucw, theta)
    k = glue.wave_constants(E, Ebar, E_s1, E_s2, pS, pD, mc, S)
    dev = E.device
    G = int(E.shape[0])
    lin = torch.empty((4, G, S), device=dev, dtype=torch.float32)
    _lib.call("kb_lin_consts", k["dl"].data_ptr(), k["ebar"].data_ptr(), k["mc"].data_ptr(), k["e"].data_ptr(),
              k["sl1"].data_ptr(), k["sl2"].data_ptr(), G * S, lin[0].data_ptr(), lin[1].data_ptr(),
              lin[2].data_ptr(), lin[3].data_ptr(), _lib.stream_handle(dev))
    k4 = None
    lay = tree.tour_layout(S)
    if lay is not None:
        k4 = torch.empty((G, lay[0], 4), device=dev, dtype=torch.float32)
        _lib.call("kb_lin_consts_tour", k["dl"].data_ptr(), k["ebar"].data_ptr(), k["mc"].data_ptr(),
                  k["e"].data_ptr(), k["sl1"].data_ptr(), k["sl2"].data_ptr(), G, S, k4.data_ptr(),
                  _lib.stream_handle(dev))
    return Prep(pS, pD, pL, mc, clp, ucw, E, E_s1, E_s2, Ebar, k, lin, k4, linear_range_flag(k))


def forward(static, theta, col_weights, *, pi_residual_out=None, prep: Prep | None = None, check_errors=True):
    """theta -> the 13 forward intermediates (same order as ``glue.solve_e_pi``) and the saved
    split reductions ``dts_wave`` [C,S] for the backward.  ``prep`` (from :func:`prepare` on the
    same theta and species tree) skips the parameter / E-step stage.  ``check_errors=False`` leaves
    the dataflow launch's error check (a host synchronisation) to the backward that follows."""
    if not supported(static):
        return glue.solve_e_pi(static, theta, col_weights, pi_residual_out=pi_residual_out), {}
    so = static.solver_options
    so.validate()
    plan = build_plan(static)
    topo = _topo(static)
    tt = topo.tt
    sh, wl = static.state_helpers, static.wave_layout
    S = int(sh["S"])
    if prep is None:
        if not glue.col_weights_uniform_for(static, col_weights):
            # the level kernels' linear-space update assumes uniform column weights (the layout of
            # every benchmark config); weighted columns take the wrapper-by-wrapper driver
            return glue.solve_e_pi(static, theta, col_weights, pi_residual_out=pi_residual_out), {}
        prep = prepare(static, theta, col_weights)
    elif prep.ucw:
        raise ValueError("the fused engine needs uniform column weights")
    pS, pD, pL, mc, clp, ucw = prep.pS, prep.pD, prep.pL, prep.mc, prep.clp, prep.ucw
    E, E_s1, E_s2, Ebar, k, lin = prep.E, prep.E_s1, prep.E_s2, prep.Ebar, prep.k, prep.lin
    dev = E.device
    G = int(E.shape[0])
    st = _lib.stream_handle(dev)
    C = int(wl["leaf_state_index"].numel())
    pi = torch.empty((C, S), device=dev, dtype=torch.float32)
    pibar = torch.empty((C, S), device=dev, dtype=torch.float32)
    row_max = torch.empty((C,), device=dev, dtype=torch.float32)
    dts = torch.empty((C, S), device=dev, dtype=torch.float32)
    leaf_state = i32(wl["leaf_state_index"])
    item_idx = i64(static.rate_item_idx)
    pDp, pSp = f32(k["pD_param"]), f32(k["pS_param"])
    prs = 0 if int(pDp.shape[0]) == 1 else S
    crs = 0 if G == 1 else S
    fallback = torch.zeros((1,), device=dev, dtype=torch.int32)
    static._fallback_rows = fallback
    rows_ptr = plan.rows.data_ptr()
    sp_ptr = plan.split_ptr.data_ptr()
    use_tour = getattr(static, "_tour_forward", True) and tt.tour is not None and prep.k4 is not None
    if use_tour and getattr(static, "_flow", True):
        fl = _flow_scratch(static, C, dev)
        _launch(static, "kb_flow_forward", 0, C, plan.row_split_ptr.data_ptr(), plan.sl_r.data_ptr(),
                plan.sr_r.data_ptr(), plan.lsp_r.data_ptr(), plan.dep0.data_ptr(), plan.ready0.data_ptr(),
                int(plan.ready0.numel()), plan.par_ptr.data_ptr(), plan.par_idx.data_ptr(), fl["queue"].data_ptr(),
                fl["remaining"].data_ptr(), fl["counters"].data_ptr(), FLOW_MAX_POLLS, pi.data_ptr(),
                pibar.data_ptr(), row_max.data_ptr(), dts.data_ptr(), _lib.ptr(pi_residual_out),
                fallback.data_ptr(), k["mc"].data_ptr(), k["dl"].data_ptr(), k["ebar"].data_ptr(),
                k["e"].data_ptr(), k["sl1"].data_ptr(), k["sl2"].data_ptr(), k["leaf"].data_ptr(), pDp.data_ptr(),
                pSp.data_ptr(), prs, crs, tt.parent.data_ptr(), tt.child1.data_ptr(), tt.child2.data_ptr(),
                topo.pre.data_ptr(), topo.pre_end.data_ptr(), tt.jumps.data_ptr(), tt.K, item_idx.data_ptr(),
                leaf_state.data_ptr(), tt.tour.data_ptr(), prep.k4.data_ptr(), 0, _lib.ptr(prep.force_log_dev),
                _lib.ptr(start_order(plan, "forward", _forward_ctas(S))
                         if getattr(static, "_forward_static_order", _one_family(static)) else None),
                int(so.pi_iters), S, st)
        note_flow_error(static, fl)
        if check_errors:
            check_flow_errors(static)
        roots = pi[wl["root_row_ids"]]
        out = (E, E_s1, E_s2, Ebar, roots, pi, pibar, row_max, pS, pD, pL, mc, clp)
        return out, {"dts_wave": dts}
    for L in range(plan.n_levels):
        a, b = plan.level_ptr[L], plan.level_ptr[L + 1]
        if b == a:
            continue
        _launch(static, "kb_level_forward", L, rows_ptr + 4 * a, sp_ptr + 8 * a, b - a, plan.sl.data_ptr(),
                  plan.sr.data_ptr(), plan.lsp.data_ptr(), pi.data_ptr(), pibar.data_ptr(), pi.data_ptr(),
                  pibar.data_ptr(), row_max.data_ptr(), dts.data_ptr(), _lib.ptr(pi_residual_out),
                  fallback.data_ptr(), k["mc"].data_ptr(), k["dl"].data_ptr(), k["ebar"].data_ptr(),
                  k["e"].data_ptr(), k["sl1"].data_ptr(), k["sl2"].data_ptr(), k["leaf"].data_ptr(),
                  lin[0].data_ptr(), lin[1].data_ptr(), lin[2].data_ptr(), lin[3].data_ptr(), pDp.data_ptr(),
                  pSp.data_ptr(), prs, crs, f32(clp).data_ptr(), int(ucw), tt.parent.data_ptr(),
                  tt.child1.data_ptr(), tt.child2.data_ptr(), topo.pre.data_ptr(), topo.pre_end.data_ptr(),
                  tt.jumps.data_ptr(), tt.K, item_idx.data_ptr(), leaf_state.data_ptr(), tt.packed_pad.data_ptr(),
                  _lib.ptr(tt.tour if use_tour else None), _lib.ptr(prep.k4 if use_tour else None),
                  int(prep.force_log), int(so.pi_iters), S, st)
    roots = pi[wl["root_row_ids"]]
    out = (E, E_s1, E_s2, Ebar, roots, pi, pibar, row_max, pS, pD, pL, mc, clp)
    return out, {"dts_wave": dts}


# Bound on one dataflow wait (polls of ~0.1-0.2 us each): far above any legitimate wait, so a
# broken dependency structure ends the launch with an error instead of hanging the GPU.
FLOW_MAX_POLLS = 1 << 25


def note_flow_error(static, fl) -> None:
    """Fold a dataflow launch's error flag (set when a wait gave up) into the static's device-side
    error word, without a host synchronisation; check_flow_errors reads it."""
    err = getattr(static, "_flow_err", None)
    if err is None or err.device != fl["counters"].device:
        err = static._flow_err = torch.zeros((1,), device=fl["counters"].device, dtype=torch.int32)
    err.bitwise_or_(fl["counters"][2:3])


def check_flow_errors(static) -> None:
    """Raise if a dataflow launch on ``static`` gave up a wait, or an E-adjoint solve whose check was
    deferred did not converge, since the last check (one host synchronisation).  The backward
    checks at its end; the forward at its end unless its caller defers the check to the backward
    that follows (``check_errors=False``)."""
    err = getattr(static, "_flow_err", None)
    if err is not None and int(err.item()) != 0:
        err.zero_()
        static._pending_e_adjoint = []
        raise RuntimeError("a dataflow wait gave up (dependency counts inconsistent); the results are invalid")
    glue.check_pending_e_adjoint(static)


def _flow_scratch(static, C, dev) -> dict:
    """Device scratch of the dataflow schedule (cached on the static)."""
    fl = getattr(static, "_flow_scratch", None)
    if fl is None or int(fl["queue"].numel()) != C or fl["queue"].device != dev:
        fl = {"queue": torch.empty((C,), device=dev, dtype=torch.int32),
              "remaining": torch.empty((C,), device=dev, dtype=torch.int32),
              "counters": torch.zeros((3,), device=dev, dtype=torch.int32)}
        static._flow_scratch = fl
    return fl


# Largest [2N, S] fp32 edge-row scratch the deterministic backward allocates (bytes); a static
# whose splits need more (a large family batch chunk) keeps the atomic adds into the adjoint rows.
EDGE_ROWS_MAX_BYTES = 16 << 30


def _edge_scratch(static, plan, C, S, dev):
    """The deterministic backward's scratch (cached on the static), or None: when it is switched
    off (``static._deterministic_backward = False``: the children's adjoint rows then take atomic
    adds, 73.0 ms against 77.8 ms for the config-3 backward), or when the edge rows would exceed
    ``EDGE_ROWS_MAX_BYTES``.  Returns the edge rows ``[2N, S]`` (row 2i / 2i+1: split i's
    contribution to its left / right child) and the CSR of each row's incoming edges
    (``in_ptr [C+1]``, ``in_edge [2N]`` ascending).  If the edge rows cannot be allocated (a GPU
    shared with other work), the static switches to the atomic form."""
    N = int(plan.n_splits)
    if not getattr(static, "_deterministic_backward", True) or N == 0 or 2 * N * S * 4 > EDGE_ROWS_MAX_BYTES:
        return None
    ed = getattr(static, "_edge_scratch", None)
    if ed is not None and ed["rows"].device == dev and tuple(ed["rows"].shape) == (2 * N, S):
        return ed
    try:
        rows = torch.empty((2 * N, S), device=dev, dtype=torch.float32)
    except torch.cuda.OutOfMemoryError:  # a GPU shared with other work: keep the atomic form
        static._deterministic_backward = False
        return None
    child = torch.stack([plan.sl_r.to(dev), plan.sr_r.to(dev)], dim=1).reshape(-1)  # edge 2i + side
    order = torch.sort(child, stable=True).indices  # by child row, ascending edge id within a row
    in_ptr = torch.zeros((C + 1,), device=dev, dtype=torch.int64)
    in_ptr[1:] = torch.cumsum(torch.bincount(child, minlength=C), dim=0)
    ed = {"rows": rows, "in_ptr": in_ptr, "in_edge": order.to(torch.int32)}
    static._edge_scratch = ed
    return ed


def new_grad_slots(static, dev) -> torch.Tensor:
    """Zeroed fp64 per-CTA accumulators ``[n_slots, 8, NTV]`` of the backward's column sums
    (rows: pD, pS, mt, E, Ebar, E_s1, E_s2, col)."""
    S = int(static.state_helpers["S"])
    bd, vpt = tree.engine_width(S)
    return torch.zeros((_backward_ctas(S, dev), 8, bd * vpt), device=dev, dtype=torch.float64)


_BWD_CTAS: dict = {}


def _backward_ctas(S, dev) -> int:
    """Resident backward CTAs on ``dev`` for S columns (one fp64 slot each)."""
    import ctypes
    key = (S, torch.device(dev).index)
    if key not in _BWD_CTAS:
        with torch.cuda.device(dev):
            n = ctypes.c_int(0)
            _lib.call("kb_backward_ctas", S, ctypes.byref(n))
            _BWD_CTAS[key] = int(n.value)
    return _BWD_CTAS[key]


def grad_accumulators_from(E, S, acc8) -> glue.GradAccumulators:
    """``GradAccumulators`` from the reduced column sums ``acc8`` [8, >=S] (any float dtype)."""
    g = glue.GradAccumulators(E, S, E.device)
    for j, name in enumerate(("pD", "pS", "mt", "E", "Ebar", "E_s1", "E_s2")):
        getattr(g, name)[0].copy_(acc8[j, :S])
    g.col.copy_(acc8[7, :S])
    return g


@torch.no_grad()
def backward(static, theta, col_weights, saved, *, v_out=None, slots=None, finish=True, check_errors=True):
    """(forward intermediates) -> (grad_theta, grad_col); uses ``saved["dts_wave"]`` when the
    forward was run by this engine, otherwise recomputes the split reductions.

    ``slots`` (from :func:`new_grad_slots`) accumulates the column sums into caller-owned fp64
    accumulators, so several chunks of a family batch add into one set; with ``finish=False``
    the E-adjoint / theta VJP and the dataflow error check (:func:`check_flow_errors`) are left
    to the caller and ``None`` is returned.  ``check_errors=False`` also leaves the check (one host
    synchronisation at the end) to the caller, e.g. once after a loop of solves."""
    if not supported(static):
        return glue.implicit_grad(static, theta, col_weights, saved)
    so = static.solver_options
    if so.self_loop_solver != "neumann":
        return glue.implicit_grad(static, theta, col_weights, saved)
    plan = build_plan(static)
    topo = _topo(static)
    tt = topo.tt
    sh, wl = static.state_helpers, static.wave_layout
    Pi, Pibar, row_max = f32(saved["pi_wave"]), f32(saved["pibar_wave"]), f32(saved["pibar_row_max"])
    C, S = int(Pi.shape[0]), int(Pi.shape[1])
    dev = Pi.device
    st = _lib.stream_handle(dev)
    E = saved["E"]
    ucw = not glue.col_weights_uniform_for(static, col_weights)
    if ucw:
        if not finish:
            raise ValueError("the fused engine needs uniform column weights")
        return glue.implicit_grad(static, theta, col_weights, saved)
    k = glue.wave_constants(E, saved["Ebar"], saved["E_s1"], saved["E_s2"], saved["log_pS"], saved["log_pD"],
                            saved["max_coupling"], S)
    G = int(E.shape[0])
    acc = torch.zeros((C, S), device=dev, dtype=torch.float32)
    roots = wl["root_row_ids"]
    acc.index_copy_(0, roots, glue.root_rhs(Pi, roots))
    if slots is None:
        slots = new_grad_slots(static, dev)
    n_slots = int(slots.shape[0])
    bd, vpt = tree.engine_width(S)
    if tuple(slots.shape[1:]) != (8, bd * vpt) or slots.dtype != torch.float64:
        raise ValueError("grad slots must be float64 [n_slots, 8, NTV] (engine.new_grad_slots)")
    dts = saved.get("dts_wave")
    leaf_state = i32(wl["leaf_state_index"])
    item_idx = i64(static.rate_item_idx)
    pDp, pSp = f32(k["pD_param"]), f32(k["pS_param"])
    prs = 0 if int(pDp.shape[0]) == 1 else S
    crs = 0 if G == 1 else S
    thr = float(so.adjoint_pruning_threshold)
    side_thr = float(so.pibar_side_threshold)
    rows_ptr = plan.rows.data_ptr()
    sp_ptr = plan.split_ptr.data_ptr()
    clp = f32(saved["col_log_probs"])
    if getattr(static, "_flow", True):
        fl = _flow_scratch(static, C, dev)
        ed = _edge_scratch(static, plan, C, S, dev)
        edge_args = (None,) * 3 if ed is None else (ed["rows"], ed["in_ptr"], ed["in_edge"])
        _launch(static, "kb_flow_backward", 0, C, plan.row_split_ptr.data_ptr(), plan.sl_r.data_ptr(),
                plan.sr_r.data_ptr(), plan.lsp_r.data_ptr(), plan.dep_b.data_ptr(), plan.ready_b.data_ptr(),
                int(plan.ready_b.numel()), plan.child_ptr.data_ptr(), plan.child_idx.data_ptr(),
                fl["queue"].data_ptr(), fl["remaining"].data_ptr(), fl["counters"].data_ptr(), FLOW_MAX_POLLS,
                Pi.data_ptr(), Pibar.data_ptr(), row_max.data_ptr(), _lib.ptr(dts), acc.data_ptr(),
                _lib.ptr(v_out), slots.data_ptr(), n_slots, thr, int(not so.use_adjoint_pruning), side_thr,
                int(side_thr > 0.0), int(so.neumann_terms), k["mc"].data_ptr(), k["dl"].data_ptr(),
                k["ebar"].data_ptr(), k["e"].data_ptr(), k["sl1"].data_ptr(), k["sl2"].data_ptr(),
                k["leaf"].data_ptr(), pDp.data_ptr(), pSp.data_ptr(), prs, crs, clp.data_ptr(), int(ucw),
                item_idx.data_ptr(), leaf_state.data_ptr(), tt.packed_pad.data_ptr(),
                _lib.ptr(start_order(plan, "backward", min(n_slots, C))
                         if getattr(static, "_backward_static_order", _one_family(static)) else None),
                *(_lib.ptr(t) for t in edge_args), S, st)
        note_flow_error(static, fl)
    else:
        _backward_levels(static, plan, rows_ptr, sp_ptr, Pi, Pibar, row_max, dts, acc, v_out, slots, n_slots, thr,
                         so, side_thr, k, pDp, pSp, prs, crs, clp, ucw, item_idx, leaf_state, tt, S, st)
    static._last_acc = acc
    if not finish:  # the caller checks the dataflow error word (check_flow_errors) when it is done
        return None
    out8 = torch.empty((8, S), device=dev, dtype=torch.float32)
    _lib.call("kb_reduce_grad_slots", slots.data_ptr(), n_slots, S, out8.data_ptr(), st)
    g = grad_accumulators_from(E, S, out8)
    grads = glue.e_adjoint_and_theta_vjp(static, theta, col_weights, saved, g, int(roots.numel()), ucw,
                                         check=check_errors)
    if check_errors:
        check_flow_errors(static)  # after everything is enqueued: the host never holds the GPU up
    return grads


def _backward_levels(static, plan, rows_ptr, sp_ptr, Pi, Pibar, row_max, dts, acc, v_out, slots, n_slots, thr, so,
                     side_thr, k, pDp, pSp, prs, crs, clp, ucw, item_idx, leaf_state, tt, S, st):
    """The level-by-level backward schedule (one kb_level_backward launch per level)."""
    for L in reversed(range(plan.n_levels)):
        a, b = plan.level_ptr[L], plan.level_ptr[L + 1]
        if b == a:
            continue
        _launch(static, "kb_level_backward", L, rows_ptr + 4 * a, sp_ptr + 8 * a, b - a, plan.sl.data_ptr(),
                plan.sr.data_ptr(), plan.lsp.data_ptr(), Pi.data_ptr(), Pibar.data_ptr(), row_max.data_ptr(),
                _lib.ptr(dts), acc.data_ptr(), _lib.ptr(v_out), slots.data_ptr(), n_slots, thr,
                int(not so.use_adjoint_pruning), side_thr, int(side_thr > 0.0), int(so.neumann_terms),
                k["mc"].data_ptr(), k["dl"].data_ptr(), k["ebar"].data_ptr(), k["e"].data_ptr(),
                k["sl1"].data_ptr(), k["sl2"].data_ptr(), k["leaf"].data_ptr(), pDp.data_ptr(), pSp.data_ptr(),
                prs, crs, clp.data_ptr(), int(ucw), item_idx.data_ptr(), leaf_state.data_ptr(),
                tt.packed_pad.data_ptr(), S, st)
