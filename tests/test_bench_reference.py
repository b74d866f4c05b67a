"""The reference arm's host-parallel oracle timing (``bench.parallel_oracle``) on a tiny sample:
spawned single-threaded processes, passes started together, one wall time per pass; and a
failing sample is reported as an error instead of a hang."""

import pytest

import bench


def test_parallel_oracle_runs_every_process_and_times_each_pass():
    rows, walls = bench.parallel_oracle("solve", (8, 16, 1), 2, 2)
    assert rows > 0
    assert len(walls) == 2 and all(w > 0.0 for w in walls)


def test_parallel_oracle_reports_a_failing_sample():
    with pytest.raises(RuntimeError, match="oracle sample process failed"):
        bench.parallel_oracle("hvp", (99, 1, 4), 1, 2)  # config 99 does not exist


def test_host_threads_is_bounded():
    assert 1 <= bench.host_threads() <= 64


def test_reference_interpreter_solves_on_the_cpu():
    """The reference's own runtime and Triton kernels under TRITON_INTERPRET=1 (the CPU baseline
    of the reference arm) run in a spawned process and agree with the oracle's loss."""
    from baseline import interpreter
    if interpreter.unavailable_reason():
        pytest.skip(interpreter.unavailable_reason())
    import numpy as np
    from kbench_b200 import gen
    from oracle import kb_oracle
    (res,) = interpreter.parallel(("tiny", 0, 7), 1)
    cap = gen.generate(gen.ProblemConfig("tiny", 4, 6, 3, 4, 12), seed=7, as_torch=False)
    st = dict(cap["static"])
    st["solver_options"] = cap["meta"]["solver_options"]
    loss, _ = kb_oracle.forward(st, cap["inputs"]["theta"], cap["inputs"]["col_weights"])
    assert res["rows"] == int(cap["meta"]["C"]) and res["solve_s"] > 0
    assert abs(res["loss"] - float(loss)) <= 1e-4 * abs(float(loss)), (res["loss"], float(loss))
