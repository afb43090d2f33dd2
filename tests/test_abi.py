"""The C-ABI library loads and exports every symbol include/tesm_b200.h declares (CPU)."""
import ctypes
import os
import re

from tesm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "tesm_b200.h")).read()
    return sorted(set(re.findall(r"\b(tesm_b200_\w+)\s*\(", text)))


def test_header_matches_binding_table():
    assert header_symbols() == sorted(_lib.SIGNATURES), "ctypes table and header disagree"


def test_library_exports_all_symbols():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in header_symbols():
        assert hasattr(lib, name), name


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.tesm_b200_version() >= 1
    assert isinstance(_lib.last_error(), str)


def test_argument_validation_without_gpu():
    # shape checks run before any CUDA call, so they work on a CPU-only host
    lib = _lib.load()
    rc = lib.tesm_b200_gemv_int2(None, 0, None, None, None, 0, None, 0, 1, 1, 1, None, 0, 1, None, 0, None)
    assert rc == 1 and "null pointer" in _lib.last_error()
    rc = lib.tesm_b200_quant_act(ctypes.c_void_p(16), 7, 1, 16, 16, 1e-5, ctypes.c_void_p(16), 256, 0,
                                 ctypes.c_void_p(16), None, None)
    assert rc == 2


def test_argument_counts_match_header():
    text = open(os.path.join(ROOT, "include", "tesm_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    for m in re.finditer(r"\b(tesm_b200_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S):
        name, params = m.group(1), m.group(2).strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert n == len(_lib.SIGNATURES[name]), f"{name}: header has {n} params, ctypes table {len(_lib.SIGNATURES[name])}"
