"""The C-ABI library loads and exports every entry point the header declares (no GPU calls)."""

import os
import re

from loopspec_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "loopspec_engine.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ls_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("ls_create", "ls_load_weight", "ls_finalize", "ls_prefill", "ls_cycle", "ls_retain",
              "ls_generate", "ls_destroy", "ls_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from loopspec_b200.build import build
    build()
    lib = _lib.lib()
    bound = {name for name, _, _ in _lib.SIGNATURES}
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in bound, f"{name} has no ctypes signature"
    assert lib.ls_version().decode().startswith("loopspec-b200")


def test_invalid_arguments_fail_cleanly_without_gpu():
    lib = _lib.lib()
    assert lib.ls_finalize(None) == _lib.LS_EINVAL
    assert lib.ls_destroy(None) == _lib.LS_EINVAL
