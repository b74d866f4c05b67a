"""GPU parity of the exact-Hessian HVP (``kbench_b200.hvp.make_exact_hvp`` over the
``kb_wave_backward_so`` / ``kb_dts_backward_so`` / ``kb_e_step_backward_so`` kernels) against the
reference's own HVP (golden fixtures) and the CPU oracle, plus each second-order kernel against
its oracle restatement.

Tolerance: the HVP and its tangent cotangents are signed accumulations over every wave, compared
with ``assert_close_vec`` (per element rel 1e-4 of the vector's largest entry plus abs 1e-6, and
norm-wise rel 1e-4)."""

import numpy as np
import pytest
import torch

from _util import GOLDEN, assert_close_vec, load_golden, oracle_static
from kbench_b200 import gen, runtime
from oracle import kb_oracle as O
from oracle import kb_oracle_hvp as OH
from oracle import kb_oracle_tangent as OT

pytestmark = pytest.mark.gpu
NAMES = sorted(p.stem for p in (GOLDEN / "hvp").glob("*.npz"))
DEBUG = ("d_gE", "d_gpD", "d_gpS", "d_gmc", "d_gEbar", "d_gEs1", "d_gEs2", "dq_E", "dwE")


def close_vec(name, got, ref):
    assert_close_vec(name, got, ref)


def _gpu_problem(cap, out, cuda):
    capt = gen.to_torch(cap)
    static = runtime.make_static(capt, cuda)
    theta = capt["inputs"]["theta"].to(cuda)
    cw = capt["inputs"]["col_weights"].to(cuda)
    sv = {k: torch.as_tensor(np.asarray(out[k])).to(cuda) for k in runtime.FORWARD_SAVED_NAMES if k in out}
    return static, theta, cw, sv


@pytest.mark.parametrize("name", NAMES)
def test_hvp_vs_reference_golden(name, cuda):
    from kbench_b200.hvp import make_exact_hvp
    cap, out = load_golden(name)
    hv = dict(np.load(GOLDEN / "hvp" / f"{name}.npz"))
    static, theta, cw, sv = _gpu_problem(cap, out, cuda)
    dbg: dict = {}
    hvp = make_exact_hvp(static, theta, cw, sv, debug_out=dbg)
    k = 0
    while f"u{k}" in hv:
        hu = hvp(torch.from_numpy(hv[f"u{k}"]).to(cuda))
        torch.cuda.synchronize()
        for key in DEBUG:
            close_vec(f"{key}[{k}]", dbg[key].cpu().numpy(), hv[f"{key}{k}"])
        close_vec(f"Hu[{k}]", hu.cpu().numpy(), hv[f"hu{k}"])
        k += 1
    assert k >= 1


WIDE = {
    "S511": gen.ProblemConfig("hvp511", 256, 16, 3, 6, 0, solver_options=dict(gen.CONFIGS[2].solver_options)),
    "S4095": gen.ProblemConfig("hvp4095", 2048, 16, 3, 6, 0, solver_options=dict(gen.CONFIGS[3].solver_options)),
}


@pytest.mark.parametrize("name", sorted(WIDE))
def test_hvp_wide_vs_oracle(name, cuda):
    """The config-2 and config-3 species tree widths on a small family, GPU against the oracle at
    the oracle's forward state."""
    from kbench_b200.hvp import make_exact_hvp
    cap = gen.generate(WIDE[name], seed=515, as_torch=False)
    st = oracle_static(cap)
    theta, cw = cap["inputs"]["theta"], cap["inputs"]["col_weights"]
    _, saved = O.forward(st, theta, cw)
    for k in ("E", "E_s1", "E_s2", "Ebar"):  # the runtime's item-row shape [1,S]
        saved[k] = np.asarray(saved[k]).reshape(1, -1)
    static, theta_d, cw_d, sv = _gpu_problem(cap, saved, cuda)
    u = np.random.default_rng(3).standard_normal(3 * theta.shape[0]).astype(np.float32)
    ref = OH.hvp(st, theta, cw, saved, u)
    got = make_exact_hvp(static, theta_d, cw_d, sv)(torch.from_numpy(u).to(cuda))
    close_vec("Hu", got.cpu().numpy(), ref)


@pytest.mark.parametrize("name", ["small_s1000"])
def test_second_order_kernels_vs_oracle(name, cuda):
    """wave_so / dts_so / e_step_so on one wave of a fixture along the reference tangent."""
    from kbench_b200 import tree
    from kbench_b200.kernels.dts_so import dts_backward_so
    from kbench_b200.kernels.e_step_so import e_step_backward_so
    from kbench_b200.kernels.wave_so import wave_backward_so
    cap, out = load_golden(name)
    st = oracle_static(cap)
    theta = cap["inputs"]["theta"]
    tg = dict(np.load(GOLDEN / "tangent" / f"{name}.npz"))
    _, dpi, dpibar, dc = OT.jvp_root_scores(st, theta, tg["v0"], out, self_iters=int(tg["self_iters"]))
    cache = OH.point_cache(st, theta, cap["inputs"]["col_weights"], out)
    wave = next(w for w in cache["waves"] if w["has_splits"] and w["W"] > 1)
    tr = O.Tree(st["state_helpers"])
    sv = {k: np.asarray(out[k], dtype=np.float32) for k in out}
    Pi, Pib, rm = sv["pi_wave"], sv["pibar_wave"], sv["pibar_row_max"]
    E = sv["E"].reshape(-1); Eb = sv["Ebar"].reshape(-1); Es1 = sv["E_s1"].reshape(-1); Es2 = sv["E_s2"].reshape(-1)
    pS = sv["log_pS"].reshape(-1); pD = sv["log_pD"].reshape(-1); pL = sv["log_pL"].reshape(-1)
    mc = sv["max_coupling"].reshape(-1)
    consts = {"dl": (1.0 + pD + E).astype(np.float32), "ebar": Eb, "e": E, "sl1": (pS + Es2).astype(np.float32),
              "sl2": (pS + Es1).astype(np.float32), "mc": mc}
    ws, W, meta, v = wave["ws"], wave["W"], wave["meta"], wave["v"]
    d_dts = OT.dts_tangent(Pi, Pib, dpi, dpibar, meta, pD, pS, dc["dpd_param"], dc["dps_param"], wave["dts_r"], tr)
    C, S = Pi.shape
    rng = np.random.default_rng(4)
    d_rhs = rng.standard_normal((C, S)).astype(np.float32)
    ref = OH.wave_backward_so(Pi, dpi, Pib, dpibar, v, ws, W, rm, consts, dc, tr, dts_r=wave["dts_r"], d_dts=d_dts,
                              d_rhs=d_rhs)
    T = lambda x: torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.float32))).to(cuda)  # noqa: E731
    sh = {k: (torch.as_tensor(np.asarray(v_)).to(cuda) if not isinstance(v_, (int, float)) else v_)
          for k, v_ in st["state_helpers"].items()}
    c1, c2, par, mad = sh["node_child1"], sh["node_child2"], sh["node_parent"], int(sh["max_ancestor_depth"])
    row = lambda x: T(np.asarray(x).reshape(1, -1))  # noqa: E731
    item_idx = torch.zeros((C,), dtype=torch.int64, device=cuda)
    leaf = torch.full((C,), -1, dtype=torch.int32, device=cuda)
    got = wave_backward_so(T(Pi), T(dpi), T(Pib), T(dpibar), T(v), ws, W, S, T(rm), row(mc), row(consts["dl"]),
                           row(dc["dDL"]), row(Eb), row(dc["dEbar"]), row(E), row(dc["dE"]), row(consts["sl1"]),
                           row(dc["dSL1"]), row(consts["sl2"]), row(dc["dSL2"]), T(sv["col_log_probs"]), c1, c2, par,
                           mad, T(wave["dts_r"]), T(d_dts), leaf_state_idx=leaf, leaf_logp=row(pS),
                           dleaf_logp=row(dc["dleaf"]), item_idx=item_idx, has_leaf_term=False, d_rhs=T(d_rhs))
    for i, nm in enumerate(("d_Av", "d_aw0", "d_aw1", "d_aw2", "d_aw345", "d_aw3", "d_aw4")):
        close_vec(f"wave_so {nm}", got[i].cpu().numpy(), ref[i])
    # dts_so
    bufs = [np.zeros((C, S), np.float32)] + [np.zeros(S, np.float32) for _ in range(4)]
    OH.dts_backward_so(Pi, dpi, Pib, dpibar, v, ws, meta, pD, pS, dc["dpd_param"], dc["dps_param"], mc, dc["dMC"], rm,
                       tr, *bufs)
    gb = [torch.zeros((C, S), device=cuda)] + [torch.zeros((1, S), device=cuda) for _ in range(3)] + \
        [torch.zeros((S,), device=cuda)]
    meta_d = {k: (torch.as_tensor(np.asarray(x)).to(cuda) if k in ("sl", "sr", "reduce_idx", "log_split_probs") else x)
              for k, x in meta.items()}
    dts_backward_so(T(Pi), T(dpi), T(Pib), T(dpibar), T(v), ws, meta_d, S, row(pD), row(pS), row(dc["dpd_param"]),
                    row(dc["dps_param"]), row(mc), row(dc["dMC"]), T(sv["col_log_probs"]), c1, c2, par, mad, T(rm),
                    item_idx, *gb)
    for nm, g, r in zip(("d_rhs", "d_gpD", "d_gpS", "d_gmt", "d_gcol"), gb, bufs):
        close_vec(f"dts_so {nm}", g.cpu().numpy(), r)
    # e_step_so
    g_new, g_eb = rng.standard_normal(S).astype(np.float32), rng.standard_normal(S).astype(np.float32)
    raw = dc["raw"]
    ref_e = OH.e_step_backward_so(E, E, Es1, Es2, Eb, pS, pD, pL, tr, g_new, g_eb, raw["dE"], raw["dE"], raw["dE_s1"],
                                  raw["dE_s2"], raw["dEbar"], raw["dlog_pS"], raw["dlog_pD"], raw["dlog_pL"])
    got_e = e_step_backward_so(row(E), row(E), row(Es1), row(Es2), row(Eb), row(pS), row(pD), row(pL),
                               T(sv["col_log_probs"]), par, c1, c2, mad, row(g_new), None, None, row(g_eb),
                               row(raw["dE"]), row(raw["dE"]), row(raw["dE_s1"]), row(raw["dE_s2"]),
                               row(raw["dEbar"]), row(raw["dlog_pS"]), row(raw["dlog_pD"]), row(raw["dlog_pL"]), None)
    for nm, g, r in zip(("d_grad_E", "d_grad_pS", "d_grad_pD", "d_grad_pL", "d_grad_mc", "d_grad_col"), got_e, ref_e):
        close_vec(f"e_step_so {nm}", g.cpu().numpy(), r)


@pytest.mark.parametrize("name", NAMES)
def test_hvp_cuda_graph_replays_match(name, cuda):
    """graph=True: one HVP captured into a CUDA graph and replayed per direction gives the same H u
    as the eager driver, for each direction in turn (the captured input buffer is refreshed)."""
    from kbench_b200.hvp import make_exact_hvp
    cap, out = load_golden(name)
    hv = dict(np.load(GOLDEN / "hvp" / f"{name}.npz"))
    static, theta, cw, sv = _gpu_problem(cap, out, cuda)
    eager = make_exact_hvp(static, theta, cw, sv)
    graphed = make_exact_hvp(static, theta, cw, sv, graph=True)
    for k in (0, 1, 0):
        u = torch.from_numpy(hv[f"u{k}"]).to(cuda)
        close_vec(f"graph Hu[{k}]", graphed(u).cpu().numpy(), eager(u).cpu().numpy())
        close_vec(f"graph Hu[{k}] vs reference", graphed(u).cpu().numpy(), hv[f"hu{k}"])


@pytest.mark.parametrize("name", NAMES)
def test_hvp_engine_tangent_matches_wave_tangent(name, cuda):
    """On a primal state from the fused forward (which carries its split reductions), the HVP's
    tangent forward runs on the engine's level launches; it must give the HVP of the wave-by-wave
    tangent sweep on the same state."""
    from kbench_b200.hvp import make_exact_hvp
    cap, _ = load_golden(name)
    hv = dict(np.load(GOLDEN / "hvp" / f"{name}.npz"))
    capt = gen.to_torch(cap)
    static = runtime.make_static(capt, cuda)
    theta = capt["inputs"]["theta"].to(cuda)
    cw = capt["inputs"]["col_weights"].to(cuda)
    _, sv = runtime.run_forward(static, theta, cw)
    u = torch.from_numpy(hv["u0"]).to(cuda)
    out = {}
    for engine_tangent in (True, False):
        static._hvp_engine_tangent = engine_tangent
        out[engine_tangent] = make_exact_hvp(static, theta, cw, sv)(u).cpu().numpy()
    close_vec("Hu engine vs wave tangent", out[True], out[False])
