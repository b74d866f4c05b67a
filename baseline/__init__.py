"""Harness for the reference baselines: the reference install (``reference``) and the full-size
comparisons with its Triton path (``parity``)."""
