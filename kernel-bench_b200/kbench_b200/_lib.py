"""ctypes binding of ``libkb_solver.so`` (the C ABI declared in ``include/kb_solver.h``).

The argument types of every ``kb_*`` entry point are derived from the header itself, so the
binding cannot drift from the declared ABI.  There is no fallback: if the shared library is
missing or fails to load, every operation raises.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libkb_solver.so"
HEADER = PKG.parent.parent / "include" / "kb_solver.h"

KB_OK, KB_ERR_ARG, KB_ERR_LAUNCH, KB_ERR_SIZE = 0, 1, 2, 3
KB_MAX_S = 8192

_CTYPES = {
    "int": ctypes.c_int,
    "long long": ctypes.c_longlong,
    "float": ctypes.c_float,
    "double": ctypes.c_double,
}

_lib = None

# Launch accounting: every kb_* call that enqueues device work increments LAUNCHES[name]
# (kb_abi_version and argument-only failures excluded).  Read by bench.py to report how many
# of this library's kernels ran inside a timed region.
LAUNCHES: dict = {}
_NO_LAUNCH = {"kb_abi_version", "kb_tour_layout", "kb_backward_layout", "kb_backward_ctas", "kb_build_workspace",
              "kb_build_emit_scratch", "kb_plan_workspace", "kb_forward_ctas", "kb_list_schedule"}


def parse_header(text: str | None = None) -> dict[str, list]:
    """Return ``{name: [ctypes arg types]}`` for every ``int kb_*(...)`` declaration."""
    if text is None:
        text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"\bint\s+(kb_\w+)\s*\(([^)]*)\)\s*;", text):
        name, args = m.group(1), m.group(2).strip()
        types = []
        if args and args != "void":
            for a in args.split(","):
                a = " ".join(a.split())
                if "*" in a:
                    types.append(ctypes.c_void_p)
                    continue
                base = re.sub(r"\b(const|unsigned)\b", "", a).strip()
                base = " ".join(base.split()[:-1])  # drop the parameter name
                if base not in _CTYPES:
                    raise ValueError(f"unsupported C type {base!r} in {name}")
                types.append(_CTYPES[base])
        decls[name] = types
    return decls


def lib():
    """Load (once) and return the shared library with argtypes set from the header."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"kbench_b200: {LIB_PATH.name} is not built (run kernel-bench_b200/kbench_b200/build.py); "
                "there is no CPU fallback")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, types in parse_header().items():
            fn = getattr(handle, name)
            fn.argtypes = types
            fn.restype = ctypes.c_int
        _lib = handle
    return _lib


def call(name: str, *args) -> None:
    """Call ``kb_<name>`` and map a non-zero status to the reference's exception types."""
    status = getattr(lib(), name)(*args)
    if status == KB_OK:
        if name not in _NO_LAUNCH:
            LAUNCHES[name] = LAUNCHES.get(name, 0) + 1
        return
    if status in (KB_ERR_ARG, KB_ERR_SIZE):
        raise ValueError(f"{name}: invalid argument or unsupported size (status {status})")
    raise RuntimeError(f"{name}: CUDA launch failed (status {status})")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
