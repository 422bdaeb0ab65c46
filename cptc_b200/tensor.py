"""Host sparse tensors: the synthetic benchmark workloads and FROSTT .tns I/O."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _native as N


@dataclass
class CooTensor:
    """Sparse tensor in coordinate form; idx[m] are 0-based uint32 indices."""

    dims: tuple
    idx: list
    vals: np.ndarray
    _keep: list = field(default_factory=list, repr=False)

    @property
    def order(self) -> int:
        return len(self.dims)

    @property
    def nnz(self) -> int:
        return int(self.vals.shape[0])

    def as_struct(self) -> N.Coo:
        """A cptc_coo view of the arrays (valid while self lives)."""
        s = N.Coo()
        s.order = self.order
        for m, d in enumerate(self.dims):
            s.dims[m] = int(d)
        s.nnz = self.nnz
        self.idx = [np.ascontiguousarray(a, dtype=np.uint32) for a in self.idx]
        self.vals = np.ascontiguousarray(self.vals, dtype=np.float64)
        for m in range(self.order):
            s.idx[m] = self.idx[m].ctypes.data_as(C.POINTER(C.c_uint32))
        s.vals = self.vals.ctypes.data_as(C.POINTER(C.c_double))
        return s

    def norm_sq(self) -> float:
        return float(np.dot(self.vals, self.vals))


class _CooOwner:
    """Owns a library-allocated cptc_coo; frees it when the last numpy array
    made from it is gone."""

    def __init__(self, s: N.Coo):
        self.s = s

    def __del__(self):
        try:
            N.host_lib().cptc_coo_free(C.byref(self.s))
        except Exception:  # interpreter shutdown
            pass


def _wrap(ptr, n: int, ctype, dtype, owner: _CooOwner) -> np.ndarray:
    if n == 0:
        return np.zeros(0, dtype=dtype)
    buf = (ctype * n).from_address(C.cast(ptr, C.c_void_p).value)
    buf._owner = owner  # the arrays keep the library memory alive
    return np.frombuffer(buf, dtype=dtype)


def _take(s: N.Coo) -> CooTensor:
    """Takes over a library-owned cptc_coo without copying: the numpy arrays
    view the library's arrays, which are freed with the last of them (a copy
    of a 76.9M-nonzero tensor costs seconds of first-touch page faults)."""
    n = int(s.nnz)
    dims = tuple(int(s.dims[m]) for m in range(s.order))
    owner = _CooOwner(s)
    idx = [_wrap(s.idx[m], n, C.c_uint32, np.uint32, owner) for m in range(s.order)]
    vals = _wrap(s.vals, n, C.c_double, np.float64, owner)
    return CooTensor(dims, idx, vals)


def gen_config(cfg: int, scale: float = 1.0, seed: int = 0) -> CooTensor:
    """Benchmark workload `cfg` (1..5) with round(nnz*scale) nonzeros."""
    lib = N.host_lib()
    s = N.Coo()
    rc = lib.cptc_gen_config(int(cfg), float(scale), int(seed), C.byref(s))
    if rc != 0:
        raise RuntimeError(f"cptc_gen_config: {lib.cptc_host_last_error().decode()}")
    return _take(s)


def gen_uniform(dims, nnz: int, seed: int = 0, values: str = "uniform") -> CooTensor:
    """Distinct uniform coordinates; values uniform (0,1], lognormal, normal
    or poisson (3)+1."""
    kinds = {"uniform": 0, "lognormal": 1, "normal": 2, "poisson": 3}
    lib = N.host_lib()
    d = (C.c_uint64 * len(dims))(*[int(x) for x in dims])
    s = N.Coo()
    rc = lib.cptc_gen_uniform(len(dims), d, int(nnz), int(seed), kinds[values], C.byref(s))
    if rc != 0:
        raise RuntimeError(f"cptc_gen_uniform: {lib.cptc_host_last_error().decode()}")
    return _take(s)


def read_tns(path: str, order: int = 0, cache=None) -> CooTensor:
    """Reads a FROSTT .tns file.  cache=True keeps a binary copy beside it
    (path + ".cptcbin"), a string names the copy; the copy is used while the
    text's size and modification time are those it was made from."""
    if cache:
        return read_tns_cached(path, order, None if cache is True else cache)[0]
    lib = N.host_lib()
    s = N.Coo()
    rc = lib.cptc_tns_read(str(path).encode(), int(order), C.byref(s))
    if rc != 0:
        raise RuntimeError(f"cptc_tns_read({path}) failed with {rc}")
    return _take(s)


def read_tns_cached(path: str, order: int = 0, cache_path=None) -> tuple:
    """(tensor, True if the binary cache was used)."""
    lib = N.host_lib()
    s = N.Coo()
    hit = C.c_int(0)
    cp = str(cache_path).encode() if cache_path else None
    rc = lib.cptc_tns_read_cached(str(path).encode(), int(order), cp, C.byref(s), C.byref(hit))
    if rc != 0:
        raise RuntimeError(f"cptc_tns_read_cached({path}) failed with {rc}")
    return _take(s), bool(hit.value)


def write_bin(path: str, t: CooTensor, src_size: int = 0, src_mtime_ns: int = 0) -> None:
    lib = N.host_lib()
    s = t.as_struct()
    if lib.cptc_bin_write(str(path).encode(), C.byref(s), int(src_size), int(src_mtime_ns)) != 0:
        raise RuntimeError(f"cptc_bin_write({path}): {lib.cptc_host_last_error().decode()}")


def read_bin(path: str) -> CooTensor:
    lib = N.host_lib()
    s = N.Coo()
    rc = lib.cptc_bin_read(str(path).encode(), C.byref(s), None, None)
    if rc != 0:
        raise RuntimeError(f"cptc_bin_read({path}) failed with {rc}: "
                           f"{lib.cptc_host_last_error().decode()}")
    return _take(s)


def write_tns(path: str, t: CooTensor) -> None:
    lib = N.host_lib()
    s = t.as_struct()
    if lib.cptc_tns_write(str(path).encode(), C.byref(s)) != 0:
        raise RuntimeError(f"cptc_tns_write({path}) failed")


def probe_order(path: str) -> int:
    return int(N.host_lib().cptc_tns_probe_order(str(path).encode()))

