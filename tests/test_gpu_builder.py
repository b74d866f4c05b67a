"""The static builder on the device (``kb_build_tables`` / ``kb_build_emit``) against the host
generator, which defines the layout: on the generator's own topologies the device layout must be
the generator's, array for array.

Bar: every integer array identical (rows, leaf states, items, roots, split children, reduce
indices, the ge2 CSR, counts); the fp32 split log-probabilities are the same fp64 expression
rounded to fp32, so they agree to within one fp32 ulp (CUDA's fp64 ``log2`` and the host's may
differ in the last fp64 bit, which moves the fp32 result only at a rounding boundary) -- measured
identical.  A forward on the device-built static is bitwise the forward on the host-built one.
"""

import numpy as np
import pytest
import torch

from kbench_b200 import builder, gen

pytestmark = pytest.mark.gpu

INT_KEYS = ("sl", "sr", "reduce_idx", "eq1_reduce_idx", "ge2_ptr", "ge2_parent_ids")
SCALAR_KEYS = ("start", "W", "n_eq1", "ge2_max_fanout")


def _np(x):
    return x.detach().cpu().numpy() if torch.is_tensor(x) else np.asarray(x)


def assert_same_layout(dev_static, host_static):
    a, b = dev_static["wave_layout"], host_static["wave_layout"]
    for k in ("leaf_state_index", "root_row_ids", "item_idx"):
        x, y = _np(a[k]), _np(b[k])
        assert x.dtype == y.dtype and np.array_equal(x, y), k
    assert len(a["wave_metas"]) == len(b["wave_metas"])
    ulps = 0
    for w, (ma, mb) in enumerate(zip(a["wave_metas"], b["wave_metas"])):
        assert sorted(ma) == sorted(mb), w
        for k in SCALAR_KEYS:
            if k in mb:
                assert int(ma[k]) == int(mb[k]), (w, k)
        for k in INT_KEYS:
            if k in mb:
                x, y = _np(ma[k]), _np(mb[k])
                assert x.dtype == y.dtype and np.array_equal(x, y), (w, k)
        if "log_split_probs" in mb:
            x, y = _np(ma["log_split_probs"]), _np(mb["log_split_probs"])
            assert x.dtype == np.float32 and x.shape == y.shape
            d = np.abs(x.view(np.int32).astype(np.int64) - y.view(np.int32).astype(np.int64))
            assert d.max(initial=0) <= 1, (w, int(d.max()))
            ulps += int((d > 0).sum())
    return ulps


@pytest.mark.parametrize("config,nf", [(1, None), (2, None), (4, 4)])
def test_device_layout_is_the_generators(cuda, config, nf):
    dev_cap = builder.generate(config, device=cuda, n_families=nf)
    host_cap = gen.generate(config, n_families=nf, as_torch=False)
    ulps = assert_same_layout(dev_cap["static"], host_cap["static"])
    for k in ("C", "n_waves", "max_W", "n_splits", "K_children"):
        assert dev_cap["meta"][k] == host_cap["meta"][k], k
    assert ulps == 0


def test_config3_family(cuda):
    """The single 4,096-gene family of config 3 (64 topologies, 128,282 rows)."""
    dev_cap = builder.generate(3, device=cuda)
    host_cap = gen.generate(3, as_torch=False)
    assert assert_same_layout(dev_cap["static"], host_cap["static"]) == 0
    assert dev_cap["meta"]["C"] == host_cap["meta"]["C"] == 128282


@pytest.mark.parametrize("rounds,alpha", [(0, 0.5), (1, 0.5), (3, 0.5), (2, 1.5)])
def test_amalgamation_options(cuda, rounds, alpha):
    species, topo = builder.family_topologies(1)
    static, stats = builder.build_static(topo, species, cuda, alpha=alpha, amalg_rounds=rounds)
    ref, ref_stats = builder.host_reference(topo, species, alpha=alpha, amalg_rounds=rounds)
    assert assert_same_layout(static, ref) == 0
    assert stats["n_splits"] == ref_stats["n_splits"] and stats["K_children"] == ref_stats["K_children"]


def test_full_tables_are_retried(cuda):
    species, topo = builder.family_topologies(4, n_families=2)
    cl, sl = builder.default_caps(topo["n_topologies"], topo["leaf_hash"].shape[1])
    # 2^(cl-3) clade and 2^(sl-4) split slots hold fewer than one family's ~16k clades / ~41k splits
    static, stats = builder.build_static(topo, species, cuda, caps=(cl - 3, sl - 4))
    ref, _ = builder.host_reference(topo, species)
    assert assert_same_layout(static, ref) == 0
    got = stats["table_caps_log2"]
    assert got[0] > cl - 3 and got[1] > sl - 4


def test_malformed_topology_is_reported(cuda):
    """An out-of-range child index is caught by the kernels' bounds checks and reported."""
    species, topo = builder.family_topologies(1)
    bad = dict(topo)
    bad["left"] = topo["left"].copy()
    G = topo["leaf_hash"].shape[1]
    bad["left"][3, G + 5] = 10 ** 6
    with pytest.raises(ValueError, match="malformed"):
        builder.build_static(bad, species, cuda)


def test_solve_on_device_static(cuda):
    """The forward on the device-built static is bitwise the forward on the host-built one; the
    gradients agree to the engine's own run-to-run spread (fp32 atomics into child adjoint rows)."""
    from kbench_b200 import runtime
    dev_cap = builder.generate(2, device=cuda)
    host_cap = gen.generate(2)
    out = []
    for cap in (dev_cap, host_cap):
        st = runtime.make_static(cap, cuda)
        theta = cap["inputs"]["theta"].to(cuda)
        cw = cap["inputs"]["col_weights"].to(cuda)
        loss, saved = runtime.run_forward(st, theta, cw)
        g = runtime.run_backward(st, theta, cw, saved)
        out.append((loss, saved, g))
    (l0, s0, g0), (l1, s1, g1) = out
    assert torch.equal(l0, l1)
    for k in ("pi_wave", "pibar_wave", "pibar_row_max", "E"):
        assert torch.equal(s0[k], s1[k]), k
    for a, b in zip(g0, g1):
        assert float((a - b).norm()) <= 1e-6 * float(b.norm()) + 1e-12


@pytest.mark.parametrize("config,nf", [(2, None), (4, 8)])
def test_device_schedule_is_the_host_schedule(cuda, config, nf):
    """The engine's schedule built on the device (kb_plan_build, from the builder's flat split
    arrays) equals the host build_plan of the same layout, array for array."""
    import dataclasses
    from types import SimpleNamespace
    from kbench_b200 import engine, runtime
    cap = builder.generate(config, device=cuda, n_families=nf)
    st = runtime.make_static(cap, cuda)
    dp = engine.build_plan(st)
    hp = engine.build_plan(SimpleNamespace(wave_layout=st.wave_layout))  # no flat arrays: host path
    assert dp.level_of is None and hp.level_of is not None
    for f in dataclasses.fields(hp):
        if f.name == "level_of":
            continue
        a, b = getattr(dp, f.name), getattr(hp, f.name)
        if torch.is_tensor(b):
            assert a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b), f.name
        else:
            assert a == b, f.name


def test_device_built_family_batch(cuda):
    """A family batch (config 4, two chunks) on device-built layouts and schedules: the same chunks
    as the host generator, the same loss, gradients within the engine's run-to-run spread."""
    from kbench_b200 import batch
    dev_chunks, timing = builder.generate_chunks(4, 0, 6, 4, device=cuda)
    host_chunks = batch.build_chunks(4, 0, 6, 4, workers=1)
    assert len(dev_chunks) == len(host_chunks) == 2 and timing["device_build_s"] > 0
    for a, b in zip(dev_chunks, host_chunks):
        assert assert_same_layout(a["static"], b["static"]) == 0
        assert a["meta"]["C"] == b["meta"]["C"] and a["meta"]["family_offset"] == b["meta"]["family_offset"]
    theta = torch.from_numpy(host_chunks[0]["inputs"]["theta"]).to(cuda)
    cw = torch.from_numpy(host_chunks[0]["inputs"]["col_weights"]).to(cuda)
    res = [batch.FamilyBatch(c, 6, batch.EngineSolver(cuda)).step(theta, cw) for c in (dev_chunks, host_chunks)]
    assert torch.equal(res[0].loss, res[1].loss)
    for a, b in ((res[0].grad_theta, res[1].grad_theta), (res[0].grad_col, res[1].grad_col)):
        assert float((a - b).norm()) <= 1e-6 * float(b.norm()) + 1e-12
