"""ctypes wrapper of the CPU oracle (oracle/cptc_oracle.cpp).

TEST INFRASTRUCTURE ONLY: a host restatement of the reference's CP-ALS /
MTTKRP arithmetic, used by tests/ as the checker and by bench.py's CPU
baseline.  The engine never imports it.  Build with ``make -C oracle``
(also done by __graft_entry__.build()).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SO = HERE / "_build" / "liboracle.so"

_lib = None

U64P = C.POINTER(C.c_uint64)
U32PP = C.POINTER(C.POINTER(C.c_uint32))
DPP = C.POINTER(C.POINTER(C.c_double))
DP = C.POINTER(C.c_double)


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return SO


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not SO.exists():
            build()
        L = C.CDLL(str(SO))
        L.or_mttkrp.argtypes = [C.c_int, U64P, C.c_uint64, U32PP, DP, C.c_int, DPP, C.c_int, DP,
                                C.c_int]
        L.or_mttkrp_hybrid3.argtypes = [U64P, C.c_uint64, U32PP, DP, C.c_int, DPP, C.c_int,
                                        C.c_double, C.c_int, DP, C.c_int]
        L.or_partition_stats3.argtypes = [U64P, C.c_uint64, U32PP, C.c_double, C.c_int, DP]
        L.or_cadr_perm.argtypes = [C.c_uint64, C.c_uint64, C.POINTER(C.c_uint32),
                                   C.POINTER(C.c_int)]
        L.or_init_factors3.argtypes = [U64P, C.c_int, DPP]
        L.or_cp_als3.argtypes = [U64P, C.c_uint64, U32PP, DP, C.c_int, C.c_int, C.c_double,
                                 C.c_int, C.c_int, DP, DP, DPP, C.c_int]
        L.or_reorder.argtypes = [C.c_int, U64P, C.c_uint64, U32PP, C.c_int, C.c_int, C.c_uint64,
                                 C.POINTER(C.POINTER(C.c_uint32))]
        L.or_mttkrp_units.argtypes = [C.c_int, U64P, C.c_uint64, U32PP, DP, C.c_int, DPP,
                                      C.POINTER(C.c_int), C.c_int, C.c_double, DP, C.c_int]
        L.or_cp_als_generic.argtypes = [C.c_int, U64P, C.c_uint64, U32PP, DP, C.c_int, C.c_int,
                                        C.c_uint, C.c_int, C.c_int, C.c_uint64, C.c_double,
                                        C.c_int, DP, DP, DPP, C.c_int]
        _lib = L
    return _lib


class _Args:
    """Keeps the ctypes views of a CooTensor alive for one call."""

    def __init__(self, t):
        self.idx = [np.ascontiguousarray(a, dtype=np.uint32) for a in t.idx]
        self.vals = np.ascontiguousarray(t.vals, dtype=np.float64)
        self.dims = (C.c_uint64 * len(t.dims))(*[int(d) for d in t.dims])
        self.ip = (C.POINTER(C.c_uint32) * len(self.idx))(
            *[a.ctypes.data_as(C.POINTER(C.c_uint32)) for a in self.idx])
        self.vp = self.vals.ctypes.data_as(DP)
        self.nnz = len(self.vals)


def _fptrs(F):
    F = [np.ascontiguousarray(f, dtype=np.float64) for f in F]
    return F, (C.POINTER(C.c_double) * len(F))(*[f.ctypes.data_as(DP) for f in F])


def mttkrp(t, factors, mode: int, threads: int = 1) -> np.ndarray:
    a = _Args(t)
    R = factors[0].shape[1]
    F, fp = _fptrs(factors)
    out = np.zeros((t.dims[mode], R))
    rc = lib().or_mttkrp(len(t.dims), a.dims, a.nnz, a.ip, a.vp, R, fp, mode,
                         out.ctypes.data_as(DP), threads)
    assert rc == 0
    return out


def mttkrp_hybrid3(t, factors, mode: int, thr: float = 0.03, sm_count: int = 148,
                   threads: int = 1):
    """Order-3 hybrid MTTKRP on coordinates as given (TF32 tiles + FP64)."""
    a = _Args(t)
    R = factors[0].shape[1]
    F, fp = _fptrs(factors)
    out = np.zeros((t.dims[mode], R))
    nt = lib().or_mttkrp_hybrid3(a.dims, a.nnz, a.ip, a.vp, R, fp, mode, thr, sm_count,
                                 out.ctypes.data_as(DP), threads)
    assert nt >= 0
    return out, nt


def partition_stats3(t, thr: float = 0.03, sm_count: int = 148) -> dict:
    a = _Args(t)
    out = (C.c_double * 5)()
    lib().or_partition_stats3(a.dims, a.nnz, a.ip, thr, sm_count, out)
    return {"dense_nnz": int(out[0]), "sparse_nnz": int(out[1]), "tiles": int(out[2]),
            "cutoff": int(out[3]), "avg_fill": out[4]}


def cadr_perm(dim: int, idx: np.ndarray) -> np.ndarray:
    idx = np.ascontiguousarray(idx, dtype=np.uint32)
    out = np.empty(dim, dtype=np.int32)
    lib().or_cadr_perm(dim, len(idx), idx.ctypes.data_as(C.POINTER(C.c_uint32)),
                       out.ctypes.data_as(C.POINTER(C.c_int)))
    return out


def init_factors3(dims, R: int):
    F = [np.empty((int(d), R)) for d in dims]
    d = (C.c_uint64 * 3)(*[int(x) for x in dims])
    _, fp = _fptrs(F)
    lib().or_init_factors3(d, R, fp)
    return F


def cp_als3(t, R: int, iters: int, thr: float = 0.03, path: str = "fp64",
            sm_count: int = 148, threads: int = 1, want_factors: bool = False):
    """Reference order-3 CP-ALS; returns (fits, lambda, factors or None)."""
    a = _Args(t)
    fits = np.zeros(iters)
    lam = np.zeros(R)
    F = [np.zeros((int(d), R)) for d in t.dims] if want_factors else None
    fp = _fptrs(F)[1] if want_factors else None
    if want_factors:
        F = [np.ascontiguousarray(f) for f in F]
        fp = (C.POINTER(C.c_double) * 3)(*[f.ctypes.data_as(DP) for f in F])
    rc = lib().or_cp_als3(a.dims, a.nnz, a.ip, a.vp, R, iters, thr, 1 if path == "tf32" else 0,
                          sm_count, fits.ctypes.data_as(DP), lam.ctypes.data_as(DP), fp, threads)
    assert rc >= 0
    return fits, lam, F


def reorder(t, kind: str = "hits", rounds: int = 3, sample: int = 8_000_000):
    kinds = {"none": 0, "cadr": 1, "hits": 2}
    a = _Args(t)
    ranks = [np.empty(int(d), dtype=np.uint32) for d in t.dims]
    rp = (C.POINTER(C.c_uint32) * len(ranks))(*[r.ctypes.data_as(C.POINTER(C.c_uint32))
                                                 for r in ranks])
    lib().or_reorder(len(t.dims), a.dims, a.nnz, a.ip, kinds[kind], rounds, sample, rp)
    return ranks


def cp_als_generic(t, R: int, iters: int, seed: int = 42, reorder: str = "default",
                   rounds: int = 3, sample: int = 8_000_000, dense_thr: float = 0.03,
                   solver: str = "chol", threads: int = 1, want_factors: bool = False):
    kinds = {"none": 0, "cadr": 1, "hits": 2}
    if reorder == "default":
        reorder = "hits" if len(t.dims) >= 4 else "cadr"
    a = _Args(t)
    fits = np.zeros(iters)
    lam = np.zeros(R)
    F = [np.zeros((int(d), R)) for d in t.dims] if want_factors else None
    fp = None
    if want_factors:
        fp = (C.POINTER(C.c_double) * len(F))(*[f.ctypes.data_as(DP) for f in F])
    rc = lib().or_cp_als_generic(len(t.dims), a.dims, a.nnz, a.ip, a.vp, R, iters, seed,
                                 kinds[reorder], rounds, sample, dense_thr,
                                 1 if solver in ("pinv", "svd") else 0, fits.ctypes.data_as(DP),
                                 lam.ctypes.data_as(DP), fp, threads)
    assert rc >= 0
    return fits, lam, F
