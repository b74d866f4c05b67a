"""The warm-started solve (``initial_v``) and the gradient targets (``self_loop_grad_targets``) of
``wave_backward_uniform_fused`` against the reference's own pristine kernels.

``tests/golden/make_wave_options.py`` recorded one backward call of the reference's glue (24 rows,
S = 31, a seeded third of the rows made inactive) and the pristine wrapper's outputs for each
option case.  Here the same arguments go through this project's wrapper on the GPU; compared:
``v_k`` (every row: active rows by tolerance, inactive rows exactly ``initial_v`` where it is
given), the six buckets or their absence, the in-place ``grad_col_log_probs`` and gradient
targets, and the last-increment output (value, or None where the reference gives None).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import GOLDEN, assert_close, assert_close_vec

FILE = GOLDEN / "wave_options_s64.pt"


def _golden():
    return torch.load(FILE, weights_only=False)


def _to(o, dev):
    if torch.is_tensor(o):
        return o.to(dev)
    if isinstance(o, dict):
        return {k: _to(v, dev) for k, v in o.items()}
    if isinstance(o, (list, tuple)):
        return type(o)(_to(v, dev) for v in o)
    return o


def test_golden_targets_are_the_bucket_column_sums():
    """The recorded reference semantics, on the CPU: the targets of the warm-started case grew by
    the column sums of the same solve's buckets (the ``initial_v`` case returns them)."""
    g = _golden()
    aw = [t.double() for t in g["cases"]["initial_v"]["aw"]]
    c = g["cases"]["initial_v_targets"]
    pre = [t.double() for t in c["extra"]["self_loop_grad_targets"][0]]
    post = [t.double() for t in c["targets_post"]]
    want = [aw[0], aw[3], aw[0] + aw[2], aw[1], aw[5], aw[4], aw[2]]
    for i in range(7):
        assert_close_vec(f"target {i}", (post[i] - pre[i]).numpy(), want[i].sum(0).numpy(), rtol=1e-5, atol=1e-6)
    v0 = g["cases"]["initial_v_zero_terms"]["v_k"]
    assert torch.equal(v0, g["cases"]["initial_v_zero_terms"]["extra"]["initial_v"])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["initial_v", "initial_v_zero_terms", "targets_vector", "targets_scalar",
                                  "initial_v_targets"])
def test_wave_backward_option_matches_reference(case, cuda):
    from kbench_b200.kernels.wave_backward import wave_backward_uniform_fused
    g = _golden()
    rec = g["cases"][case]
    args, kw = _to(g["args"], cuda), _to(g["kwargs"], cuda)
    extra = _to(rec["extra"], cuda)
    if "self_loop_grad_targets" in extra:
        vals, vec = extra["self_loop_grad_targets"]
        extra["self_loop_grad_targets"] = (*[v.clone() for v in vals], vec)
    kw.update(extra)
    res = wave_backward_uniform_fused(*args, **kw)
    torch.cuda.synchronize()
    assert len(res) == (8 if rec["has_last"] else 7)
    mask = g["kwargs"]["active_mask"].numpy()
    v = res[0].cpu().numpy()
    ref_v = rec["v_k"].numpy()
    assert_close(f"{case} v_k (active rows)", v[mask], ref_v[mask])
    if "initial_v" in rec["extra"]:
        assert np.array_equal(v[~mask], rec["extra"]["initial_v"].numpy()[~mask])
    if rec["aw"] is None:
        assert all(t is None for t in res[1:7])
    else:
        for i, (got, want) in enumerate(zip(res[1:7], rec["aw"])):
            assert_close(f"{case} aw[{i}]", got.cpu().numpy(), want.numpy())
    if rec["grad_col_post"] is not None:
        assert_close_vec(f"{case} grad_col", kw["grad_col_log_probs"].cpu().numpy(), rec["grad_col_post"].numpy())
    if "targets_post" in rec:
        for i, (got, want) in enumerate(zip(kw["self_loop_grad_targets"][:7], rec["targets_post"])):
            assert_close_vec(f"{case} target {i}", got.cpu().numpy(), want.numpy())
    if rec["has_last"]:
        if rec["last_rel"] is None:
            assert res[7] is None
        else:
            assert_close(f"{case} last increment", res[7].cpu().numpy()[mask], rec["last_rel"].numpy()[mask])


@pytest.mark.gpu
def test_wave_backward_option_errors(cuda):
    from kbench_b200.kernels.wave_backward import wave_backward_uniform_fused
    g = _golden()
    args, kw = _to(g["args"], cuda), _to(g["kwargs"], cuda)
    W, S = g["W"], g["S"]
    with pytest.raises(ValueError, match="GMRES self-loop solve does not support initial_v"):
        wave_backward_uniform_fused(*args, **{**kw, "self_loop_solver": "gmres",
                                              "initial_v": torch.zeros((W, S), device=cuda)})
    with pytest.raises(ValueError, match="does not match wave scratch shape"):
        wave_backward_uniform_fused(*args, **{**kw, "initial_v": torch.zeros((W + 1, S), device=cuda)})
    bad = tuple(torch.zeros(S, device=cuda) for _ in range(6)) + (torch.zeros(S, device=cuda, dtype=torch.float64),
                                                                   True)
    with pytest.raises(ValueError, match="self_loop_grad_targets"):
        wave_backward_uniform_fused(*args, **{**kw, "self_loop_grad_targets": bad})


def test_oracle_options_match_reference_golden():
    """The CPU oracle's warm start and gradient targets (``oracle/kb_oracle.py`` ``wave_backward``)
    against the same pristine-kernel outputs, on the CPU."""
    from oracle import kb_oracle as O
    g = _golden()
    a, kw = g["args"], g["kwargs"]
    W, S, ws = g["W"], g["S"], int(a[2])
    n = lambda t: t.detach().numpy()  # noqa: E731
    tree = O.Tree({"S": S, "node_parent": n(kw["node_parent"]), "node_child1": n(a[14]), "node_child2": n(a[15]),
                   "node_subtree_start": np.zeros(S), "node_subtree_end": np.zeros(S),
                   "max_ancestor_depth": kw["max_ancestor_depth"], "unnorm_row_max": np.zeros(1),
                   "compact_level_ptr": n(kw["compact_level_ptr"]),
                   "compact_level_parents": n(kw["compact_level_parents"]),
                   "compact_level_child1": n(kw["compact_level_child1"]),
                   "compact_level_child2": n(kw["compact_level_child2"])})
    assert a[5] is None and int(kw["item_idx"].abs().max()) == 0  # the leaf wave of one family
    consts = {k: n(a[i]).reshape(S) for k, i in (("dl", 8), ("ebar", 9), ("e", 10), ("sl1", 11), ("sl2", 12))}
    mask = n(kw["active_mask"]).astype(bool)
    for case, rec in g["cases"].items():
        ex = rec["extra"]
        gc = n(g["kwargs"]["grad_col_log_probs"]).copy()
        targets = None
        if "self_loop_grad_targets" in ex:
            vals, vec = ex["self_loop_grad_targets"]
            targets = (*[n(v).copy() for v in vals], bool(vec))
        out = O.wave_backward(n(a[0]), n(a[1]), n(kw["pibar_row_max"]), ws, W, None, n(a[6]), consts,
                              n(a[13]), tree, neumann_terms=int(ex.get("neumann_terms", kw["neumann_terms"])),
                              leaf_state=n(kw["leaf_state_idx"])[ws:ws + W].astype(np.int64),
                              leaf_logp=n(kw["leaf_logp"]).reshape(S), active=mask, grad_col=gc,
                              initial_v=None if "initial_v" not in ex else n(ex["initial_v"]),
                              grad_targets=targets)
        assert_close(f"{case} v_k", out[0][mask], n(rec["v_k"])[mask])
        if "initial_v" in ex:
            assert np.array_equal(out[0][~mask], n(ex["initial_v"])[~mask])
        if rec["aw"] is None:
            assert all(t is None for t in out[1:])
        else:
            for i, (got, want) in enumerate(zip(out[1:], rec["aw"])):
                assert_close(f"{case} aw[{i}]", got, n(want))
        assert_close_vec(f"{case} grad_col", gc, n(rec["grad_col_post"]))
        if targets is not None:
            for i, want in enumerate(rec["targets_post"]):
                assert_close_vec(f"{case} target {i}", targets[i], n(want))
