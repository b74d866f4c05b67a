"""The allocation-free E fixed point (``kb_e_fixed_point_noalloc``) against the allocating entry
point (``kb_e_fixed_point``), through the C ABI.

Some callers of this library cannot allocate device memory where they need the E-step: a host
that manages every device byte through its own pool and forbids driver allocations, or one that
must not trigger an allocation (and its possible synchronisation) at that point.  The no-alloc
entry point serves them by taking its iteration buffer from a fixed device array inside the
library; this test checks it returns what the regular entry point returns, on consecutive calls
that reuse the shared array.  The file is named to be collected last.
"""

import pytest
import torch

from kbench_b200 import _lib, gen, glue, runtime, tree

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-6


def _problem(cfg, device, seed=None):
    cap = gen.generate(cfg, seed=seed)
    static = runtime.make_static(cap, device)
    theta = cap["inputs"]["theta"].to(device)
    cw = cap["inputs"]["col_weights"].to(device)
    pS, pD, pL, mc, clp, ucw = glue.solve_parameters(static, theta, cw)
    sh = static.state_helpers
    tt = tree.tables(sh["node_parent"], sh["node_child1"], sh["node_child2"], int(sh["max_ancestor_depth"]))
    S = int(sh["S"])
    rows = [t.reshape(1, S).contiguous() for t in (pS, pD, pL, mc)]
    return dict(S=S, rows=rows, clp=clp.contiguous(), tt=tt, ucw=int(ucw),
                max_iter=static.solver_options.e_max_iter, tol=static.solver_options.e_tol)


def _outputs(S, device, G=1):
    return [torch.empty((G, S), device=device) for _ in range(4)] + [torch.zeros(G, dtype=torch.int32, device=device)]


def _args(pb, E0, outs):
    tt = pb["tt"]
    pS, pD, pL, mc = pb["rows"]
    G = int(pS.shape[0])
    return [E0.data_ptr(), outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(), outs[3].data_ptr(),
            pS.data_ptr(), pD.data_ptr(), pL.data_ptr(), mc.data_ptr(), pb["clp"].data_ptr(), tt.parent.data_ptr(),
            tt.child1.data_ptr(), tt.child2.data_ptr(), tt.jumps.data_ptr(), tt.K, pb["S"], G, int(pb["max_iter"]),
            float(pb["tol"]), pb["ucw"], outs[4].data_ptr(), _lib.stream_handle()]


def _allocating(pb, E0, device):
    G = int(E0.shape[0])
    outs = _outputs(pb["S"], device, G)
    tmp = torch.empty((G, pb["S"]), device=device)
    args = _args(pb, E0, outs)
    args.insert(2, tmp.data_ptr())  # E_tmp follows E_out
    _lib.call("kb_e_fixed_point", *args)
    return outs


def _no_alloc(pb, E0, device):
    outs = _outputs(pb["S"], device, int(E0.shape[0]))
    _lib.call("kb_e_fixed_point_noalloc", *_args(pb, E0, outs))
    return outs


def _assert_same(got, ref):
    for g, r in zip(got[:4], ref[:4]):
        fin = torch.isfinite(r)
        assert torch.equal(torch.isfinite(g), fin)
        assert torch.all((g[fin] - r[fin]).abs() <= ATOL + RTOL * r[fin].abs())
    assert torch.equal(got[4], ref[4])


def test_no_alloc_matches_allocating_entry_point(cuda):
    for cfg in (1, 2):
        pb = _problem(cfg, cuda)
        E0 = torch.full((1, pb["S"]), -1.0, device=cuda)
        ref = _allocating(pb, E0, cuda)
        first = _no_alloc(pb, E0, cuda)    # first call on this device also performs the set-up
        second = _no_alloc(pb, E0, cuda)   # reuses the shared array holding the previous contents
        torch.cuda.synchronize()
        _assert_same(first, ref)
        _assert_same(second, ref)


def test_no_alloc_item_rows_and_both_buffer_parities(cuda):
    """Several item rows (each its own fixed point, G x S elements of the shared array) and
    iteration caps of 3 and 4, so that the final iterate ends in either half of the array's
    ping-pong pair, then the problem's own cap; two calls in a row each time."""
    base = _problem(1, cuda)
    S, G = base["S"], 4
    shift = torch.linspace(-0.3, 0.3, G, device=cuda).reshape(G, 1)
    pS, pD, pL, mc = base["rows"]
    rows = [pS.expand(G, S).contiguous(), (pD + shift).contiguous(), (pL - shift).contiguous(),
            mc.expand(G, S).contiguous()]
    E0 = torch.full((G, S), -1.0, device=cuda)
    for cap_iters in (3, 4, int(base["max_iter"])):
        pb = dict(base, rows=rows, max_iter=cap_iters)
        ref = _allocating(pb, E0, cuda)
        first = _no_alloc(pb, E0, cuda)
        second = _no_alloc(pb, E0, cuda)
        torch.cuda.synchronize()
        _assert_same(first, ref)
        _assert_same(second, ref)


def test_no_alloc_rejects_sizes_beyond_its_capacity():
    with pytest.raises(ValueError):
        # 4095 columns x 17 item rows > 65536 elements: rejected before any device work
        _lib.call("kb_e_fixed_point_noalloc", *([None] * 14), 0, 4095, 17, 10, 1e-6, 0, None, None)
