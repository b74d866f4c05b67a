"""Host-side parameter addressing of the split-reduction wrappers against the reference (no GPU).

* Backward (``dts_cross_backward_accum_fused``): every shape / item-indexing combination is
  classified as the reference's layout contract classifies it
  (``kbench/core/kernels/_dts_layout_contract.py`` ``dts_backward_param_layout``, imported from the
  installed reference in ``baseline/_ref``), the rejected ones with the reference's ValueError.
* Forward (``compute_dts_forward`` / ``compute_dts_tangent``): the value each (item, column) reads
  equals the reference's ``_load_rate`` addressing (``dts_fused.py:11-16`` with the wrapper's
  ``by_state`` / ``row_stride`` at ``:193-194``), restated here."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
from baseline import reference  # noqa: E402
from kbench_b200.kernels._common import state_rows  # noqa: E402
from kbench_b200.kernels.wave_backward import _dts_backward_layout, _param_ref  # noqa: E402

S_VALUES = (5, 7)
G = 3


def _shapes(S):
    return [(), (1,), (1, 1), (S,), (G,), (S, 1), (G, 1), (1, S), (G, S), (S, S), (G, 2), (G, S, 1), (2, 2, 2)]


def _contract():
    if not (reference.REF / "kbench").is_dir():
        pytest.skip("reference not installed in baseline/_ref")
    if str(reference.REF) not in sys.path:
        sys.path.insert(0, str(reference.REF))
    from kbench.core.kernels import _dts_layout_contract as c  # pure host code, no Triton
    return c


@pytest.mark.parametrize("S", S_VALUES)
@pytest.mark.parametrize("item_indexed", [False, True])
def test_backward_layouts_follow_the_reference_contract(S, item_indexed):
    c = _contract()
    want_of = {0: (0, 0), 1: (0, 1), 2: (1, 0), 3: None}
    for shape in _shapes(S):
        try:
            code = int(c.dts_backward_param_layout(shape, S=S, item_indexed=item_indexed).code)
        except ValueError:
            code = None
        got = _dts_backward_layout(shape, S, item_indexed)
        if code is None:
            assert got is None, shape
            with pytest.raises(ValueError, match="fused DTS backward path"):
                _param_ref(torch.zeros(shape), S=S, item_indexed=item_indexed, device=torch.device("cpu"))
            continue
        if code == 3:  # one row per item; a single row is shared
            assert got == ((0 if shape[0] == 1 else S), 1), shape
        else:
            assert got == want_of[code], (shape, code, got)


@pytest.mark.parametrize("S", S_VALUES)
def test_forward_addressing_matches_the_reference_load_rate(S):
    rng = np.random.default_rng(7)
    for shape in [(1,), (1, 1), (S,), (G,), (G, 1), (1, S), (G, S), (S, S)]:
        t = torch.from_numpy(rng.standard_normal(shape).astype(np.float32))
        flat = t.reshape(-1).numpy()
        by_state = t.ndim == 2 and int(t.shape[1]) != 1
        row_stride = 0 if int(t.shape[0]) == 1 else int(t.stride(0))
        rows, rs = state_rows(t, S)
        got = rows.reshape(-1).numpy()
        n_items = 1 if int(t.shape[0]) == 1 else int(t.shape[0])
        for item in range(n_items):
            for s in range(S):
                want = flat[item * row_stride + (s if by_state else 0)]
                assert got[item * rs + s] == want, (shape, item, s)
    with pytest.raises(ValueError):
        state_rows(torch.zeros((G, 2)), S)
