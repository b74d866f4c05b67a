"""Static builder on the device: gene-tree topologies -> the ``captured`` wave layout.

The solver consumes a static layout (rows = clades ordered by size, per-wave split arrays) that the
reference reads from an external capture (``kbench/runtime.py:47-60``); the preprocessing that
made it is not part of the reference (``capture/capture.py:17-18``).  :mod:`kbench_b200.gen`
builds it on the host (clade amalgamation in Python dictionaries); this module builds the same
layout on the GPU through ``kb_build_tables`` / ``kb_build_emit`` (``csrc/kb_builder.cu``), for
batches of families:

    cap = builder.generate(4, n_families=128, device="cuda")      # like gen.generate(4, ...)
    static, stats = builder.build_static(topo, species, "cuda")   # from given topologies

The result equals :func:`gen.assemble_static` over :func:`gen.family_from_topologies` of the same
topologies: every integer array identical, the fp32 split log-probabilities from the same fp64
expression (``log2((count + alpha) / (n_obs + alpha * n_splits))``) rounded to fp32.  The static's
arrays are device tensors (per-wave entries are views of flat arrays); the species tree's
``state_helpers`` come from the host generator.  Only the gene-topology sampling
(:func:`gen.sample_topologies`, a seeded host random process) stays on the host.
"""

from __future__ import annotations

import math
import multiprocessing as mp
import os

import numpy as np
import torch

from . import _lib, gen

STATUS_BITS = {1: "clade table full", 2: "split table full", 4: "reserved hash value (~0)",
               8: "malformed topology", 16: "missing clade", 32: "count overflow"}


def default_caps(n_topologies: int, n_genes: int) -> tuple[int, int]:
    """log2 of the per-family clade / split table capacities: >= 1.25 x the clade instances (every
    internal node of every topology plus the gene leaves) and >= 3 x the observed splits (room for
    the amalgamation's additions; a full table is retried larger)."""
    inst = n_topologies * (n_genes - 1)
    cl = max(4, math.ceil(math.log2(1.25 * (inst + n_genes))))
    sl = max(4, math.ceil(math.log2(3.0 * max(inst, 1))))
    return cl, sl


def _sample_unit(args):
    cfg, species, seed = args
    return gen.sample_topologies(cfg, species, seed)


def family_topologies(config, *, seed: int | None = None, n_families: int | None = None, family_offset: int = 0,
                      workers: int = 1) -> tuple[dict, dict]:
    """(species tree, stacked topologies) of families ``[family_offset, family_offset + n)`` of a
    benchmark config, sampled exactly as :func:`gen.generate` samples them (family ``f`` from seed
    ``seed + 1 + f``).  Topologies: int32 ``left`` / ``right`` [F*T, 2G-1], int32 ``root``
    [F*T], uint64 ``leaf_hash`` [F, G], int64 ``leaf_species`` [F, G].  ``workers`` > 1 samples
    families in a ``spawn`` process pool."""
    cfg = gen.CONFIGS[config] if isinstance(config, int) else config
    cfg_id = config if isinstance(config, int) else 0
    seed = 1000 * cfg_id if seed is None else int(seed)
    nf = cfg.n_families if n_families is None else int(n_families)
    species = gen.make_species_tree(cfg.n_species, seed)
    jobs = [(cfg, species, seed + 1 + family_offset + f) for f in range(nf)]
    if workers > 1 and nf > 1:
        with mp.get_context("spawn").Pool(min(workers, nf)) as pool:
            fams = pool.map(_sample_unit, jobs, chunksize=max(1, nf // (4 * workers)))
    else:
        fams = [_sample_unit(j) for j in jobs]
    return species, stack_topologies(fams)


def stack_topologies(fams: list[dict]) -> dict:
    """Stack per-family :func:`gen.sample_topologies` outputs into the builder's batch arrays."""
    T, NN = fams[0]["left"].shape
    return {
        "left": np.concatenate([f["left"] for f in fams]).astype(np.int32).reshape(-1, NN),
        "right": np.concatenate([f["right"] for f in fams]).astype(np.int32).reshape(-1, NN),
        "root": np.concatenate([f["root"] for f in fams]).astype(np.int32),
        "leaf_hash": np.stack([np.asarray(f["leaf_hash"], dtype=np.uint64) for f in fams]),
        "leaf_species": np.stack([np.asarray(f["leaf_species"], dtype=np.int64) for f in fams]),
        "n_topologies": int(T),
    }


def _dev(a, device, dtype):
    if torch.is_tensor(a):
        return a.to(device=device, dtype=dtype).contiguous()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint64:
        a = a.view(np.int64)  # raw 64-bit words; the kernels read them as unsigned
    return torch.from_numpy(a).to(device=device, dtype=dtype)


def _status_message(status: int) -> str:
    return ", ".join(v for k, v in STATUS_BITS.items() if status & k) or f"status {status}"


def build_static(topo: dict, species: dict, device, *, alpha: float = 0.5, amalg_rounds: int = 2,
                 caps: tuple[int, int] | None = None, max_retries: int = 4) -> tuple[dict, dict]:
    """The ``static`` part of a captured problem (and its stats, as :func:`gen.assemble_static`
    returns them) built on ``device`` from stacked topologies (:func:`stack_topologies`;
    numpy arrays or tensors).  Raises ``ValueError`` on malformed input."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("the static builder runs on a CUDA device")
    leaf_hash = topo["leaf_hash"]
    F, G = (int(x) for x in leaf_hash.shape)
    left_np = topo["left"]
    NN = int(left_np.shape[-1])
    if NN != 2 * G - 1:
        raise ValueError(f"topologies have {NN} nodes, expected 2G-1 = {2 * G - 1}")
    TT = int(np.prod(left_np.shape[:-1]))
    if TT % F:
        raise ValueError("topology count is not a multiple of the family count")
    T = TT // F
    left = _dev(topo["left"], dev, torch.int32).reshape(TT, NN)
    right = _dev(topo["right"], dev, torch.int32).reshape(TT, NN)
    root = _dev(topo["root"], dev, torch.int32).reshape(TT)
    lh = _dev(leaf_hash, dev, torch.int64).reshape(F, G)
    lsp_host = _dev(topo["leaf_species"], dev, torch.int64).reshape(F, G)
    cl, sl = caps if caps is not None else default_caps(T, G)
    stream = _lib.stream_handle(dev)
    sizes = np.zeros(5, dtype=np.int64)
    for _ in range(max_retries + 1):
        nbytes = np.zeros(1, dtype=np.int64)
        _lib.call("kb_build_workspace", F, T, G, cl, sl, nbytes.ctypes.data)
        ws = torch.empty(int(nbytes[0]), dtype=torch.uint8, device=dev)
        _lib.call("kb_build_tables", _lib.ptr(left), _lib.ptr(right), _lib.ptr(root), _lib.ptr(lh), F, T, G,
                  int(amalg_rounds), float(alpha), cl, sl, _lib.ptr(ws), int(nbytes[0]), sizes.ctypes.data, stream)
        status = int(sizes[3])
        if not status:
            break
        if not status & 3:
            raise ValueError(f"static builder: {_status_message(status)}")
        # a full table (which also leaves clades missing downstream): retry with it doubled
        cl += status & 1
        sl += (status >> 1) & 1
        del ws
    else:
        raise ValueError(f"static builder: {_status_message(status)} after {max_retries} retries")
    C, N, n_waves = int(sizes[0]), int(sizes[1]), int(sizes[2])

    i32 = dict(dtype=torch.int32, device=dev)
    i64 = dict(dtype=torch.int64, device=dev)
    leaf_state = torch.empty(C, **i32)
    item_idx = torch.empty(C, **i64)
    root_rows = torch.empty(F, **i64)
    row_local = torch.empty(C, **i64)
    sl_t, sr_t, red_t = torch.empty(N, **i64), torch.empty(N, **i64), torch.empty(N, **i64)
    srow_t = torch.empty(N, **i64)
    rsp_t = torch.empty(C + 1, **i64)
    lsp_t = torch.empty(N, dtype=torch.float32, device=dev)
    ge2 = torch.empty(C + n_waves, **i64)
    table = torch.empty((n_waves, 8), **i64)
    nscr = np.zeros(1, dtype=np.int64)
    _lib.call("kb_build_emit_scratch", N, nscr.ctypes.data)
    scratch = torch.empty(int(nscr[0]), dtype=torch.uint8, device=dev)
    kout = np.zeros(2, dtype=np.int64)
    _lib.call("kb_build_emit", _lib.ptr(ws), _lib.ptr(lh), _lib.ptr(lsp_host), F, T, G, cl, sl, C, N, n_waves,
              _lib.ptr(leaf_state), _lib.ptr(item_idx), _lib.ptr(root_rows), _lib.ptr(row_local), _lib.ptr(sl_t),
              _lib.ptr(sr_t), _lib.ptr(red_t), _lib.ptr(srow_t), _lib.ptr(rsp_t), _lib.ptr(lsp_t), _lib.ptr(ge2),
              _lib.ptr(table), _lib.ptr(scratch), int(nscr[0]), kout.ctypes.data, stream)
    if int(kout[1]):
        raise ValueError(f"static builder: {_status_message(int(kout[1]))}")
    del ws, scratch
    tab = table.cpu().numpy()
    metas = []
    max_w = 0
    for w in range(n_waves):
        start, W, n1, sb, se, fan, size, g0 = (int(x) for x in tab[w])
        max_w = max(max_w, W)
        meta = {"start": start, "W": W}
        if size > 1:
            meta.update({
                "sl": sl_t[sb:se], "sr": sr_t[sb:se], "reduce_idx": red_t[sb:se], "log_split_probs": lsp_t[sb:se],
                "n_eq1": n1, "eq1_reduce_idx": row_local[start:start + n1],
                "ge2_ptr": ge2[g0:g0 + W - n1 + 1], "ge2_parent_ids": row_local[start + n1:start + W],
                "ge2_max_fanout": fan,
            })
        metas.append(meta)
    static = {
        "wave_layout": {"leaf_state_index": leaf_state, "root_row_ids": root_rows, "item_idx": item_idx,
                        "wave_metas": metas},
        "state_helpers": {k: v for k, v in species.items() if not k.startswith("_")},
        "rate_item_idx": torch.zeros(C, **i64),
        "itemwise": False,
        "statewise": True,
        # the same splits as flat row-ordered arrays: the engine builds its schedule from these on
        # the device (engine.build_plan)
        "flat_layout": {"split_row": srow_t, "sl": sl_t, "sr": sr_t, "lsp": lsp_t, "row_split_ptr": rsp_t,
                        "wave_split_ptr": [int(x) for x in tab[:, 3]] + [N]},
    }
    stats = {"C": C, "n_waves": n_waves, "max_W": max_w, "n_splits": N,
             "splits_per_internal_row": N / max(1, C - F * G), "K_children": int(kout[0]),
             "amalgamation_added": int(sizes[4]), "table_caps_log2": (cl, sl)}
    return static, stats


def _captured(cfg, cfg_id, seed, species, static, stats, nf, family_offset, solver_options):
    S = species["S"]
    so = dict(cfg.solver_options)
    if solver_options:
        so.update(solver_options)
    meta = {
        "label": cfg.name, "config": cfg_id, "seed": seed, "S": S, "C": stats["C"],
        "n_items": nf, "family_offset": family_offset, "solver_options": so,
        "theta_columns": ["log2_dup", "log2_loss", "log2_transfer"],
        **{k: stats[k] for k in ("C", "n_waves", "max_W", "n_splits", "splits_per_internal_row", "K_children")},
    }
    static["state_helpers"] = gen.to_torch(static["state_helpers"])
    inputs = {"theta": torch.from_numpy(gen.make_theta(S, seed + 7)),
              "col_weights": torch.zeros(S, dtype=torch.float32)}
    return {"meta": meta, "static": static, "inputs": inputs}


def _resolve(config, seed):
    cfg = gen.CONFIGS[config] if isinstance(config, int) else config
    cfg_id = config if isinstance(config, int) else 0
    return cfg, cfg_id, 1000 * cfg_id if seed is None else int(seed)


def generate(config, *, device, seed: int | None = None, n_families: int | None = None, family_offset: int = 0,
             solver_options: dict | None = None, workers: int = 1, alpha: float = 0.5, amalg_rounds: int = 2):
    """:func:`gen.generate` with the layout stage on the device: the same ``captured`` dictionary
    (``meta``, ``static``, ``inputs``), its static arrays device tensors."""
    cfg, cfg_id, seed = _resolve(config, seed)
    nf = cfg.n_families if n_families is None else int(n_families)
    species, topo = family_topologies(cfg, seed=seed, n_families=nf, family_offset=family_offset, workers=workers)
    static, stats = build_static(topo, species, device, alpha=alpha, amalg_rounds=amalg_rounds)
    return _captured(cfg, cfg_id, seed, species, static, stats, nf, family_offset, solver_options)


def slice_topologies(topo: dict, a: int, b: int) -> dict:
    """Families ``[a, b)`` of stacked topologies."""
    T = int(topo["n_topologies"])
    return {"left": topo["left"][a * T:b * T], "right": topo["right"][a * T:b * T], "root": topo["root"][a * T:b * T],
            "leaf_hash": topo["leaf_hash"][a:b], "leaf_species": topo["leaf_species"][a:b], "n_topologies": T}


def generate_chunks(config, f0: int, f1: int, chunk: int, *, device, seed: int | None = None, workers: int = 1,
                    solver_options: dict | None = None) -> tuple[list[dict], dict]:
    """The captured dicts of families ``[f0, f1)`` of a batched config in chunks of at most
    ``chunk`` families (what ``batch.build_chunks`` makes on the host), the layouts built on
    ``device``; returns (chunks, timings in seconds: topology sampling, device build)."""
    import time
    from .batch import chunk_ranges
    cfg, cfg_id, seed = _resolve(config, seed)
    t0 = time.perf_counter()
    species, topo = family_topologies(cfg, seed=seed, n_families=f1 - f0, family_offset=f0, workers=workers)
    t1 = time.perf_counter()
    out = []
    for a, b in chunk_ranges(f0, f1, chunk):
        static, stats = build_static(slice_topologies(topo, a - f0, b - f0), species, device)
        out.append(_captured(cfg, cfg_id, seed, species, static, stats, b - a, a, solver_options))
    torch.cuda.synchronize(device)
    return out, {"sampling_s": t1 - t0, "device_build_s": time.perf_counter() - t1}


def host_reference(topo: dict, species: dict, *, alpha: float = 0.5, amalg_rounds: int = 2) -> tuple[dict, dict]:
    """The host generator's layout of the same stacked topologies (the builder's specification)."""
    F = int(topo["leaf_hash"].shape[0])
    T = int(topo["n_topologies"]) if "n_topologies" in topo else int(topo["left"].shape[0]) // F
    fams = []
    for f in range(F):
        one = {"left": np.asarray(topo["left"][f * T:(f + 1) * T]), "right": np.asarray(topo["right"][f * T:(f + 1) * T]),
               "root": np.asarray(topo["root"][f * T:(f + 1) * T]), "leaf_hash": np.asarray(topo["leaf_hash"][f]),
               "leaf_species": np.asarray(topo["leaf_species"][f])}
        fams.append(gen.family_from_topologies(one, alpha=alpha, amalg_rounds=amalg_rounds))
    return gen.assemble_static(fams, species)


def cpu_count() -> int:
    return len(os.sched_getaffinity(0))


def main():
    """``python -m kbench_b200.builder --config 4 --families 128``: sample the topologies, build the
    static layout and the engine's schedule on the GPU once, and print the sizes and timings."""
    import argparse
    import json
    import time
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=4)
    ap.add_argument("--families", type=int, default=None)
    ap.add_argument("--workers", type=int, default=cpu_count())
    a = ap.parse_args()
    from . import engine, runtime
    dev = torch.device("cuda:0")
    species, topo = family_topologies(a.config, n_families=a.families, workers=a.workers)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    static, stats = build_static(topo, species, dev)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    cap = _captured(*_resolve(a.config, None), species, static, stats, int(topo["leaf_hash"].shape[0]), 0, None)
    st = runtime.make_static(cap, dev)
    plan = engine.build_plan(st)
    torch.cuda.synchronize()
    t2 = time.perf_counter()
    print(json.dumps({"config": a.config, "families": int(topo["leaf_hash"].shape[0]), "rows": stats["C"],
                      "splits": stats["n_splits"], "waves": stats["n_waves"], "levels": plan.n_levels,
                      "layout_s": round(t1 - t0, 4), "schedule_s": round(t2 - t1, 4)}), flush=True)


if __name__ == "__main__":
    main()
