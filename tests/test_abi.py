"""The C ABI shared library loads on the CPU host and exports every entry point the public header
declares (no device calls: these tests run without a GPU)."""

import ctypes
import re
from pathlib import Path

import pytest

from kbench_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kb_solver.h"


def test_header_parses_all_entry_points():
    decls = _lib.parse_header()
    text = re.sub(r"/\*.*?\*/", " ", HEADER.read_text(), flags=re.S)
    names = set(re.findall(r"\bint\s+(kb_\w+)\s*\(", text))
    assert names == set(decls)
    assert {"kb_wave_step", "kb_dts_forward", "kb_e_fixed_point", "kb_wave_adjoint", "kb_level_forward",
            "kb_level_backward"} <= names


def test_library_exports_every_declared_symbol():
    if not _lib.LIB_PATH.exists():
        pytest.skip("libkb_solver.so not built")
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _lib.parse_header():
        assert hasattr(handle, name), name
    lib = _lib.lib()
    assert lib.kb_abi_version() == 4


def test_invalid_sizes_are_rejected_without_a_device():
    """Argument validation happens on the host before any launch."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("libkb_solver.so not built")
    lib = _lib.lib()
    assert lib.kb_active_mask(None, 0, -1, 4, 0.0, 0, None, None) == _lib.KB_ERR_ARG
    assert lib.kb_e_step_forward(*([None] * 15), 0, 0, 1, 0, None) == _lib.KB_ERR_ARG
    with pytest.raises(ValueError):
        _lib.call("kb_active_mask", None, 0, -1, 4, 0.0, 0, None, None)


def test_tour_layout_matches_host_tables():
    """The forward tour kernel's layout in the library equals the one the host tables are built
    for (kbench_b200.tree.tour_layout), for every S up to the library maximum."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("libkb_solver.so not built")
    from kbench_b200 import tree
    lib = _lib.lib()
    ntv, nt, vf = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    for S in list(range(1, 300)) + [511, 1023, 2047, 4095, 4096, 8191]:
        st = lib.kb_tour_layout(S, ctypes.byref(ntv), ctypes.byref(nt), ctypes.byref(vf))
        want = tree.tour_layout(S)
        if want is None:
            assert st == _lib.KB_ERR_SIZE and ntv.value == 0
        else:
            assert st == _lib.KB_OK and (ntv.value, nt.value, vf.value) == want
            assert nt.value % 32 == 0 and vf.value in (2, 4, 8) and ntv.value > S


def test_backward_layout_is_whole_warps_over_the_padded_width():
    """The backward kernels' block for every S up to the library maximum: whole warps (their scans
    take lane 31 of every warp), at most 1024 threads, threads x columns = the padded width the
    host builds the column tables for (kbench_b200.tree.engine_width)."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("libkb_solver.so not built")
    from kbench_b200 import tree
    lib = _lib.lib()
    ntv, nt, v = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    for S in range(1, 8192):
        assert lib.kb_backward_layout(S, ctypes.byref(ntv), ctypes.byref(nt), ctypes.byref(v)) == _lib.KB_OK
        bd, vpt = tree.engine_width(S)
        assert ntv.value == bd * vpt == nt.value * v.value
        assert nt.value % 32 == 0 and 32 <= nt.value <= 1024 and v.value in (1, 2, 4, 8)
    for S in (8192, 8193):
        assert lib.kb_backward_layout(S, ctypes.byref(ntv), ctypes.byref(nt), ctypes.byref(v)) == _lib.KB_ERR_SIZE
