"""ctypes bindings of the native libraries (declarations in include/*.h).

libcptc_host.so — host-only: generators, .tns reader/writer, binary cache.
libcptc.so      — the CUDA engine (also exports the host symbols).

Loading fails loudly: there is no Python or CPU fallback for the engine.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"

MAX_ORDER = 8


class Coo(C.Structure):
    """struct cptc_coo (include/cptc_host.h)."""

    _fields_ = [
        ("order", C.c_int),
        ("dims", C.c_uint64 * MAX_ORDER),
        ("nnz", C.c_uint64),
        ("idx", C.POINTER(C.c_uint32) * MAX_ORDER),
        ("vals", C.POINTER(C.c_double)),
    ]


class Opts(C.Structure):
    """struct cptc_opts (include/cptc.h)."""

    _fields_ = [
        ("path", C.c_int),
        ("fill_min", C.c_double),
        ("generic", C.c_int),
        ("reorder", C.c_int),
        ("reorder_rounds", C.c_int),
        ("reorder_sample", C.c_uint64),
        ("solver", C.c_int),
        ("seed", C.c_uint32),
        ("dense_generic", C.c_int),
        ("dense_thr_generic", C.c_double),
        ("dense_inner", C.c_int * 3),
        ("verbose", C.c_int),
        ("exchange", C.c_int),
    ]


class Stats(C.Structure):
    """struct cptc_stats (include/cptc.h)."""

    _fields_ = [
        ("order", C.c_int),
        ("dims", C.c_uint64 * MAX_ORDER),
        ("nnz", C.c_uint64),
        ("rank", C.c_int),
        ("tf32_path", C.c_int),
        ("dense_nnz", C.c_uint64),
        ("sparse_nnz", C.c_uint64),
        ("dense_tiles", C.c_uint64),
        ("avg_fill", C.c_double),
        ("fill_min", C.c_double),
        ("cutoff", C.c_int),
        ("x_norm_sq", C.c_double),
        ("build_ms", C.c_double),
        ("device_bytes", C.c_uint64),
        ("fiber_mode", C.c_int * MAX_ORDER),
        ("nranks", C.c_int),
        ("rank_id", C.c_int),
        ("reorder_ms", C.c_double),
        ("local_sparse_nnz", C.c_uint64 * MAX_ORDER),
        ("local_rows", C.c_uint64 * MAX_ORDER),
        ("local_tiles", C.c_uint64 * MAX_ORDER),
        ("local_tile_words", C.c_uint64 * MAX_ORDER),
    ]


ITER_CB = C.CFUNCTYPE(None, C.c_int, C.c_double, C.c_double, C.POINTER(C.c_double), C.c_int,
                      C.c_void_p)

# Every symbol of include/cptc_host.h and include/cptc.h with its signature.
HOST_SYMBOLS = {
    "cptc_coo_free": (None, [C.POINTER(Coo)]),
    "cptc_tns_read": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(Coo)]),
    "cptc_tns_probe_order": (C.c_int, [C.c_char_p]),
    "cptc_tns_write": (C.c_int, [C.c_char_p, C.POINTER(Coo)]),
    "cptc_bin_write": (C.c_int, [C.c_char_p, C.POINTER(Coo), C.c_uint64, C.c_int64]),
    "cptc_bin_read": (C.c_int, [C.c_char_p, C.POINTER(Coo), C.POINTER(C.c_uint64),
                                C.POINTER(C.c_int64)]),
    "cptc_tns_read_cached": (C.c_int, [C.c_char_p, C.c_int, C.c_char_p, C.POINTER(Coo),
                                       C.POINTER(C.c_int)]),
    "cptc_gen_config": (C.c_int, [C.c_int, C.c_double, C.c_uint64, C.POINTER(Coo)]),
    "cptc_gen_uniform": (C.c_int, [C.c_int, C.POINTER(C.c_uint64), C.c_uint64, C.c_uint64,
                                   C.c_int, C.POINTER(Coo)]),
    "cptc_host_last_error": (C.c_char_p, []),
}

ENGINE_SYMBOLS = {
    "cptc_opts_default": (C.c_int, [C.POINTER(Opts)]),
    "cptc_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_int]),
    "cptc_destroy": (C.c_int, [C.c_void_p]),
    "cptc_last_error": (C.c_char_p, [C.c_void_p]),
    "cptc_comm_unique_id": (C.c_int, [C.POINTER(C.c_ubyte)]),
    "cptc_comm_init": (C.c_int, [C.c_void_p, C.POINTER(C.c_ubyte), C.c_int, C.c_int]),
    "cptc_load_coo": (C.c_int, [C.c_void_p, C.POINTER(Coo)]),
    "cptc_build": (C.c_int, [C.c_void_p, C.c_int, C.c_double, C.POINTER(Opts)]),
    "cptc_init_factors": (C.c_int, [C.c_void_p]),
    "cptc_set_factors": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double)]),
    "cptc_set_factors_sharded": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double)]),
    "cptc_get_factors_sharded": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double)]),
    "cptc_get_factors": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double)]),
    "cptc_get_lambda": (C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
    "cptc_mttkrp": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double)]),
    "cptc_mttkrp_timed": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "cptc_profile_mttkrp": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "cptc_profile_gather": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "cptc_launch_count": (C.c_ulonglong, []),
    "cptc_gather_peak": (C.c_int, [C.c_int, C.c_uint64, C.c_int, C.c_uint64, C.c_int,
                                   C.POINTER(C.c_double)]),
    "cptc_phase_timing": (C.c_int, [C.c_void_p, C.c_int]),
    "cptc_phase_times": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.c_int]),
    "cptc_als": (C.c_int, [C.c_void_p, C.c_int, ITER_CB, C.c_void_p]),
    "cptc_get_stats": (C.c_int, [C.c_void_p, C.POINTER(Stats)]),
    "cptc_fit_terms": (C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
    "cptc_get_relabel": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_uint32)]),
    "cptc_residual_noalloc": (C.c_int, [C.c_int, C.c_uint64, C.POINTER(C.c_void_p), C.c_void_p,
                                        C.c_int, C.POINTER(C.c_void_p), C.c_void_p, C.c_void_p,
                                        C.c_void_p]),
    "cptc_residual": (C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
}

_host = None
_engine = None


def _bind(lib: C.CDLL, table: dict) -> C.CDLL:
    for name, (res, args) in table.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def host_lib() -> C.CDLL:
    """libcptc_host.so (no CUDA needed)."""
    global _host
    if _host is None:
        path = LIB_DIR / "libcptc_host.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing: run `python -m cptc_b200.build`")
        _host = _bind(C.CDLL(str(path)), HOST_SYMBOLS)
    return _host


def engine_lib() -> C.CDLL:
    """libcptc.so, the CUDA engine.  Raises if it was not built."""
    global _engine
    if _engine is None:
        path = LIB_DIR / "libcptc.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing: run `python -m cptc_b200.build`; "
                               "the engine has no CPU fallback")
        lib = C.CDLL(str(path), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        _bind(lib, HOST_SYMBOLS)
        _engine = _bind(lib, ENGINE_SYMBOLS)
    return _engine
