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
