"""Flat (npz-friendly) serialisation of a problem (``captured`` dict) plus named outputs.

The nested ``static`` layout (wave metas are a list of dicts) is flattened to ``name -> array``
so a whole problem and its reference outputs fit one ``.npz``; :func:`unflatten_case` rebuilds
the dictionaries (numpy arrays; convert with ``gen.to_torch``).
"""

from __future__ import annotations

import json

import numpy as np

_WAVE_ARRAYS = ("sl", "sr", "reduce_idx", "log_split_probs", "eq1_reduce_idx", "ge2_ptr",
                "ge2_parent_ids")
_WAVE_INTS = ("start", "W", "n_eq1", "ge2_max_fanout")


def _np(x):
    try:
        import torch
        if torch.is_tensor(x):
            return x.detach().cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x)


def flatten_case(captured: dict, outputs: dict | None = None) -> dict:
    st = captured["static"]
    arrays = {}
    scalars = {"meta": captured["meta"], "itemwise": bool(st["itemwise"]),
               "statewise": bool(st["statewise"]), "waves": []}
    for k, v in st["state_helpers"].items():
        if isinstance(v, (int, float)) and not hasattr(v, "shape"):
            scalars[f"sh_{k}"] = v
        else:
            arrays[f"sh__{k}"] = _np(v)
    wl = st["wave_layout"]
    for k in ("leaf_state_index", "root_row_ids", "item_idx"):
        arrays[f"wl__{k}"] = _np(wl[k])
    arrays["rate_item_idx"] = _np(st["rate_item_idx"])
    for i, meta in enumerate(wl["wave_metas"]):
        ints = {k: int(meta[k]) for k in _WAVE_INTS if k in meta}
        scalars["waves"].append(ints)
        for k in _WAVE_ARRAYS:
            if k in meta:
                arrays[f"w{i}__{k}"] = _np(meta[k])
    for k, v in captured["inputs"].items():
        arrays[f"in__{k}"] = _np(v)
    for k, v in (outputs or {}).items():
        arrays[f"out__{k}"] = _np(v)
    arrays["__json__"] = np.frombuffer(json.dumps(scalars).encode(), dtype=np.uint8)
    return arrays


def unflatten_case(arrays) -> tuple[dict, dict]:
    """Inverse of :func:`flatten_case`: returns (captured, outputs) with numpy arrays."""
    scalars = json.loads(bytes(np.asarray(arrays["__json__"])).decode())
    sh = {}
    wl = {}
    inputs = {}
    outputs = {}
    rate = None
    per_wave = {}
    for name in arrays.keys() if hasattr(arrays, "keys") else arrays.files:
        if name == "__json__":
            continue
        v = np.asarray(arrays[name])
        if name.startswith("sh__"):
            sh[name[4:]] = v
        elif name.startswith("wl__"):
            wl[name[4:]] = v
        elif name.startswith("in__"):
            inputs[name[4:]] = v
        elif name.startswith("out__"):
            outputs[name[5:]] = v
        elif name == "rate_item_idx":
            rate = v
        elif name.startswith("w") and "__" in name:
            idx, key = name[1:].split("__", 1)
            per_wave.setdefault(int(idx), {})[key] = v
    for k, v in scalars.items():
        if k.startswith("sh_"):
            sh[k[3:]] = v
    metas = []
    for i, ints in enumerate(scalars["waves"]):
        m = dict(ints)
        m.update(per_wave.get(i, {}))
        metas.append(m)
    wl["wave_metas"] = metas
    captured = {
        "meta": scalars["meta"],
        "static": {"wave_layout": wl, "state_helpers": sh, "rate_item_idx": rate,
                   "itemwise": scalars["itemwise"], "statewise": scalars["statewise"]},
        "inputs": inputs,
    }
    return captured, outputs
