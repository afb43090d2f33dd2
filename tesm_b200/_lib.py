"""ctypes loader for libtesm_b200.so (the C ABI declared in include/tesm_b200.h).

The library is built in-tree (``python __graft_entry__.py`` or
``make -C tesm_b200/csrc``).  A missing library is a hard error: the b200 backend
has no fallback path.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtesm_b200.so")

_lock = threading.Lock()
_lib = None

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_float = ctypes.c_float
c_vp = ctypes.c_void_p

# name -> argument types (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "tesm_b200_version": [],
    "tesm_b200_last_error": [],
    "tesm_b200_device_status": [c_vp],
    "tesm_b200_weight_scale": [c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_float, c_vp, c_vp, c_vp, c_vp],
    "tesm_b200_pack_ternary": [c_vp, c_int, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp],
    "tesm_b200_unpack_ternary": [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp],
    "tesm_b200_quant_act": [c_vp, c_int, c_i64, c_i64, c_i64, c_float, c_vp, c_i64, c_int, c_vp, c_vp, c_vp],
    "tesm_b200_gemv_int2": [c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_int,
                            c_i64, c_vp, c_i64, c_vp],
    "tesm_b200_gemm_i8": [c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_int, c_i64,
                          c_vp, c_i64, c_vp, c_i64, c_vp],
    "tesm_b200_gemm_bf16": [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_int, c_i64, c_vp],
    "tesm_b200_scan_workspace": [c_i64, c_i64, c_i64, c_i64, c_vp],
    "tesm_b200_siso_scan": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp,
                            c_vp, c_vp, c_i64, c_vp],
    "tesm_b200_mimo_scan": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                            c_vp, c_vp, c_vp, c_i64, c_vp],
    "tesm_b200_siso_local_ent": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                                 c_float, c_float, c_float, c_vp, c_vp, c_int, c_vp],
    "tesm_b200_global_relbias": [c_vp, c_i64, c_float, c_float, c_i64, c_vp, c_vp],
    "tesm_b200_siso_global_ent": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                                  c_float, c_float, c_float, c_vp, c_vp, c_int, c_vp],
    "tesm_b200_siso_decode_step_codes": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                                         c_vp, c_vp, c_vp, c_vp, c_float, c_float, c_float, c_int, c_float,
                                         c_float, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp,
                                         c_float, c_vp],
    "tesm_b200_row_absmax": [c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_vp],
    "tesm_b200_quant_act_amax": [c_vp, c_int, c_i64, c_i64, c_i64, c_float, c_vp, c_vp, c_i64, c_int, c_vp, c_vp,
                                 c_vp],
    "tesm_b200_acc_scale": [c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_vp, c_int, c_i64, c_vp],
    "tesm_b200_combine_acc": [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64,
                              c_vp, c_int, c_i64, c_vp],
    "tesm_b200_global_ent_tc_workspace": [c_i64, c_i64, c_i64, c_i64, c_vp],
    "tesm_b200_siso_global_ent_tc": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                                     c_float, c_float, c_float, c_vp, c_vp, c_int, c_vp, c_i64, c_vp],
    "tesm_b200_mimo_local_ent": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp,
                                 c_vp, c_vp, c_float, c_float, c_float, c_int, c_vp, c_vp, c_int, c_vp],
    "tesm_b200_mimo_global_ent": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp,
                                  c_vp, c_float, c_float, c_vp, c_vp, c_vp, c_vp, c_int, c_vp],
    "tesm_b200_combine": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_int, c_vp, c_int, c_vp],
    "tesm_b200_cache_fill": [c_vp, c_int, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                             c_float, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    "tesm_b200_decode_step": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp,
                              c_vp, c_vp, c_vp, c_vp, c_float, c_float, c_float, c_vp, c_vp, c_int, c_vp, c_vp],
    "tesm_b200_embed": [c_vp, c_i64, c_i64, c_vp, c_vp, c_int, c_i64, c_vp, c_i64, c_vp, c_int, c_vp],
    "tesm_b200_add_rmsnorm_quant": [c_vp, c_int, c_vp, c_vp, c_vp, c_float, c_i64, c_i64, c_float, c_vp, c_i64,
                                    c_int, c_vp, c_vp, c_vp, c_int, c_vp],
    "tesm_b200_silu_mul": [c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_int, c_vp],
    "tesm_b200_siso_local_ent_codes": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp,
                                       c_vp, c_float, c_float, c_float, c_int, c_float, c_float, c_vp, c_i64, c_i64,
                                       c_vp, c_vp, c_vp],
    "tesm_b200_gemm_i8_combine": [c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_int, c_i64, c_i64,
                                  c_i64, c_i64, c_i64, c_vp, c_int, c_i64, c_vp],
    "tesm_b200_gemm_i8_swiglu": [c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_int, c_i64,
                                 c_vp, c_i64, c_vp],
    "tesm_b200_siso_scan_noalloc": [c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp,
                                    c_vp, c_vp, c_vp, c_vp],
}
_RESTYPES = {"tesm_b200_last_error": ctypes.c_char_p}


class TesmError(RuntimeError):
    pass


def load(path: str = LIB_PATH):
    """Load the shared library and declare every exported signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise TesmError(f"kernel_backend='b200' specified but libtesm_b200.so is not available at {path}; "
                            f"build it with `python __graft_entry__.py build`")
        lib = ctypes.CDLL(path)
        for name, argt in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argt
            fn.restype = _RESTYPES.get(name, c_int)
        _lib = lib
        return lib


def get():
    return _lib if _lib is not None else load()


def last_error() -> str:
    msg = get().tesm_b200_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str):
    if status != 0:
        raise TesmError(f"tesm_b200 {what} failed (status {status}): {last_error()}")


# number of entry-point calls that enqueue device work (bench.py reports it as gpu_launches)
launch_count = 0
_NO_LAUNCH = {"tesm_b200_version", "tesm_b200_last_error", "tesm_b200_device_status", "tesm_b200_scan_workspace"}


def call(name: str, *args):
    global launch_count
    if name not in _NO_LAUNCH:
        launch_count += 1
    check(getattr(get(), name)(*args), name)


def exported_symbols():
    return list(SIGNATURES)
