"""The C-ABI library loads and exports every function include/rdet.h
declares (no GPU needed: nothing is called)."""
import ctypes as C
import os
import re

from helpers import ROOT, rdet


def declared_functions():
    with open(os.path.join(ROOT, "include", "rdet.h")) as f:
        text = f.read()
    return re.findall(r"^\s*(?:int32_t|const char\*)\s+(rdet_\w+)\s*\(", text, re.M)


def test_header_lists_every_symbol():
    decl = declared_functions()
    assert sorted(decl) == sorted(rdet.SYMBOLS)


def test_library_exports_declared_symbols():
    L = C.CDLL(rdet.LIB_PATH)
    for name in declared_functions():
        assert hasattr(L, name), name
    assert b"sm_100a" in rdet.lib().rdet_version()


def test_no_oracle_in_product():
    # the product package never imports or links the CPU oracle
    pkg = os.path.join(ROOT, "raster-inference_b200")
    for dirpath, _, files in os.walk(pkg):
        for fn in files:
            if fn.endswith((".py", ".cu", ".cuh", ".h", ".cpp")) or fn == "Makefile":
                with open(os.path.join(dirpath, fn)) as f:
                    src = f.read()
                assert "det_oracle" not in src and "import oracle" not in src, fn
