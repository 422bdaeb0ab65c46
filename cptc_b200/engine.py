"""Python face of the CP-ALS engine (a thin ctypes layer over include/cptc.h).

Mirrors the reference's operator interface for the MTTKRP hot path:

  reference (zhixianzhu/cpTC)                      here
  ----------------------------------------------   ---------------------------
  load_tns_file / load_tns_generic                 read_tns() / Engine.load()
  compute/apply_cadr_reordering,                   Engine.build()
    partition_tensor_hybrid, build_mttkrp_views,
    fill-rate selector (src/main.cu:316-426)
  init_factors_random (src/common.cu:66-126)       Engine.init_factors()
  run_mttkrp_mode: compute_dense_mttkrp_async +    Engine.mttkrp(mode)
    compute_sparse_mttkrp_async (src/als.cu:535)
  execute_als_decomposition / run_generic_cp       Engine.als(iters)
  unpermute_factor_matrices                        Engine.factors()

Errors raise CptcError with the library's message; nothing falls back to
the CPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .tensor import CooTensor

PATHS = {"auto": 0, "tf32": 1, "fp64": 2}
REORDERS = {"default": -1, "none": 0, "cadr": 1, "hits": 2, "auto": 3}
SOLVERS = {"default": 0, "chol": 1, "cholesky": 1, "pinv": 2, "svd": 2}
EXCHANGES = {"nccl": 0, "peer": 1}


class CptcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


@dataclass
class IterReport:
    iter: int
    ms: float
    fit: float
    mode_ms: list
    phases: np.ndarray | None = None  # (order, 5) ms when phase timing is on


def default_opts() -> N.Opts:
    o = N.Opts()
    N.engine_lib().cptc_opts_default(C.byref(o))
    return o


def launch_count() -> int:
    """Kernels launched by libcptc.so since it was loaded."""
    return int(N.engine_lib().cptc_launch_count())


def gather_peak(device: int, rows: int, R: int, n: int, reps: int = 3) -> float:
    """GB/s of uniformly random R-wide FP64 row gathers from an L2-resident
    rows x R matrix with the residual kernel's row layout (cptc_gather_peak):
    the ceiling of the sparse MTTKRP's factor-row gathers on this GPU."""
    out = C.c_double(0.0)
    rc = N.engine_lib().cptc_gather_peak(int(device), int(rows), int(R), int(n), int(reps),
                                         C.byref(out))
    if rc != 0:
        raise CptcError(rc, "cptc_gather_peak failed")
    return float(out.value)


def comm_unique_id() -> bytes:
    buf = (C.c_ubyte * 128)()
    rc = N.engine_lib().cptc_comm_unique_id(buf)
    if rc != 0:
        raise CptcError(rc, "ncclGetUniqueId failed")
    return bytes(buf)


class Engine:
    """One CP-ALS context on one GPU."""

    def __init__(self, device: int = 0):
        self._lib = N.engine_lib()
        h = C.c_void_p()
        rc = self._lib.cptc_create(C.byref(h), int(device), 0)
        if rc != 0:
            raise CptcError(rc, f"cptc_create(device={device}) failed")
        self._h = h
        self._tensor = None
        self.R = 0

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.cptc_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            msg = self._lib.cptc_last_error(self._h)
            raise CptcError(rc, f"{what}: {msg.decode() if msg else ''}")

    # -- multi-GPU -------------------------------------------------------
    def comm_init(self, uid: bytes, rank: int, nranks: int) -> None:
        buf = (C.c_ubyte * 128).from_buffer_copy(uid)
        self._check(self._lib.cptc_comm_init(self._h, buf, int(rank), int(nranks)), "comm_init")

    # -- tensor and build --------------------------------------------------
    def load(self, t: CooTensor) -> None:
        self._tensor = t
        s = t.as_struct()
        self._check(self._lib.cptc_load_coo(self._h, C.byref(s)), "load")

    def build(self, R: int, threshold: float = 0.03, path: str = "auto", generic: bool = False,
              reorder: str = "default", reorder_rounds: int = 3,
              reorder_sample: int = 8_000_000, solver: str = "default", seed: int = 42,
              dense_generic: bool = True, dense_thr_generic: float = 0.03,
              dense_inner: tuple = (0, 1, 2), fill_min: float = 0.0,
              exchange: str = "nccl") -> None:
        o = default_opts()
        o.exchange = EXCHANGES[exchange]
        o.path = PATHS[path]
        o.fill_min = float(fill_min)
        o.generic = int(bool(generic))
        o.reorder = REORDERS[reorder]
        o.reorder_rounds = int(reorder_rounds)
        o.reorder_sample = int(reorder_sample)
        o.solver = SOLVERS[solver]
        o.seed = int(seed)
        o.dense_generic = int(bool(dense_generic))
        o.dense_thr_generic = float(dense_thr_generic)
        for q in range(3):
            o.dense_inner[q] = int(dense_inner[q])
        self._check(self._lib.cptc_build(self._h, int(R), float(threshold), C.byref(o)), "build")
        self.R = int(R)

    def init_factors(self) -> None:
        self._check(self._lib.cptc_init_factors(self._h), "init_factors")

    def relabel(self, mode: int) -> np.ndarray:
        """The build's relabelling of `mode`: out[old index] = new index."""
        out = np.empty(int(self._tensor.dims[mode]), dtype=np.uint32)
        self._check(self._lib.cptc_get_relabel(self._h, int(mode),
                                               out.ctypes.data_as(C.POINTER(C.c_uint32))),
                    "relabel")
        return out

    def stats(self) -> dict:
        s = N.Stats()
        self._check(self._lib.cptc_get_stats(self._h, C.byref(s)), "stats")
        out = {k: getattr(s, k) for k, _ in N.Stats._fields_}
        out["dims"] = tuple(int(s.dims[m]) for m in range(s.order))
        out["fiber_mode"] = tuple(int(s.fiber_mode[m]) for m in range(s.order))
        for k in ("local_sparse_nnz", "local_rows", "local_tiles", "local_tile_words"):
            out[k] = tuple(int(getattr(s, k)[m]) for m in range(s.order))
        return out

    # -- factors ---------------------------------------------------------
    def _dims(self):
        return self._tensor.dims

    def set_factor(self, mode: int, F: np.ndarray, sharded: bool = False) -> None:
        """Factor `mode` in the tensor's own labels.  sharded=True (collective
        on several ranks): this rank copies only its 1/G of the rows and the
        pieces are all-gathered on the GPUs."""
        F = np.ascontiguousarray(F, dtype=np.float64)
        assert F.shape == (self._dims()[mode], self.R)
        fn = self._lib.cptc_set_factors_sharded if sharded else self._lib.cptc_set_factors
        self._check(fn(self._h, int(mode), F.ctypes.data_as(C.POINTER(C.c_double))),
                    "set_factors")

    def factor(self, mode: int, out: np.ndarray = None, sharded: bool = False) -> np.ndarray:
        """Factor `mode` in the tensor's own labels.  `out`, when given, is a
        C-contiguous float64 (I_mode, R) array to fill (e.g. pinned memory).
        sharded=True fills only this rank's 1/G of the rows (the others are
        left as they are)."""
        shape = (self._dims()[mode], self.R)
        if out is None:
            out = np.zeros(shape, dtype=np.float64) if sharded else np.empty(shape, np.float64)
        elif out.shape != shape or out.dtype != np.float64 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float64 array of shape {shape}")
        fn = self._lib.cptc_get_factors_sharded if sharded else self._lib.cptc_get_factors
        self._check(fn(self._h, int(mode), out.ctypes.data_as(C.POINTER(C.c_double))),
                    "get_factors")
        return out

    def factors(self) -> list:
        return [self.factor(m) for m in range(len(self._dims()))]

    def lam(self, out: np.ndarray = None) -> np.ndarray:
        if out is None:
            out = np.empty(self.R, dtype=np.float64)
        elif out.shape != (self.R,) or out.dtype != np.float64:
            raise ValueError(f"out must be a float64 array of shape ({self.R},)")
        self._check(self._lib.cptc_get_lambda(self._h, out.ctypes.data_as(C.POINTER(C.c_double))),
                    "get_lambda")
        return out

    # -- hot path --------------------------------------------------------
    def mttkrp(self, mode: int) -> np.ndarray:
        out = np.empty((self._dims()[mode], self.R), dtype=np.float64)
        self._check(self._lib.cptc_mttkrp(self._h, int(mode),
                                          out.ctypes.data_as(C.POINTER(C.c_double))), "mttkrp")
        return out

    def mttkrp_timed(self, mode: int, reps: int = 1) -> float:
        ms = C.c_double(0.0)
        self._check(self._lib.cptc_mttkrp_timed(self._h, int(mode), int(reps), C.byref(ms)),
                    "mttkrp_timed")
        return ms.value

    def profile_mttkrp(self, mode: int, reps: int = 3) -> dict:
        """Device ms of the dense-tile kernel, the FP64 view kernel and the
        whole MTTKRP of `mode` (mean of `reps` launches each)."""
        ms = (C.c_double * 3)()
        self._check(self._lib.cptc_profile_mttkrp(self._h, int(mode), int(reps), ms),
                    "profile_mttkrp")
        return {"tiles_ms": ms[0], "sparse_ms": ms[1], "total_ms": ms[2]}

    def profile_gather(self, mode: int, reps: int = 3) -> dict:
        """Device ms per launch of a gather-only replay of the order-3 residual
        MTTKRP's memory accesses and of the kernel itself (cptc_profile_gather)."""
        ms = (C.c_double * 2)()
        self._check(self._lib.cptc_profile_gather(self._h, int(mode), int(reps), ms),
                    "profile_gather")
        return {"replay_ms": ms[0], "kernel_ms": ms[1]}

    PHASES = ("mttkrp", "inverse_wait", "solve", "exchange", "normalise")

    def set_phase_timing(self, on: bool = True) -> None:
        """Time every phase of each mode update from the next als() on."""
        self._check(self._lib.cptc_phase_timing(self._h, int(bool(on))), "phase_timing")

    def phase_times(self) -> np.ndarray:
        """(order, 5) device ms of the last finished iteration's phases, in
        the order of PHASES; empty when phase timing is off."""
        n = N.MAX_ORDER * len(self.PHASES)
        buf = (C.c_double * n)()
        got = self._lib.cptc_phase_times(self._h, buf, n)
        if got < 0:
            self._check(got, "phase_times")
        return np.array(buf[:got], dtype=np.float64).reshape(-1, len(self.PHASES))

    def fit_terms(self) -> dict:
        out = (C.c_double * 3)()
        self._check(self._lib.cptc_fit_terms(self._h, out), "fit_terms")
        return {"iprod": out[0], "model2": out[1], "fit": out[2]}

    def residual(self) -> dict:
        """Exact sum of squared errors over the stored nonzeros, ||X||^2,
        RMSE and exact fit with the current factors and lambda."""
        out = (C.c_double * 2)()
        self._check(self._lib.cptc_residual(self._h, out), "residual")
        res2, x2 = out[0], out[1]
        n = self._tensor.nnz
        return {"res_sq": res2, "x_sq": x2, "rmse": (res2 / n) ** 0.5 if n else 0.0,
                "fit": 1.0 - (max(res2, 0.0) ** 0.5) / (x2 ** 0.5) if x2 > 0 else 0.0}

    def als(self, iters: int, callback=None) -> list:
        reports = []

        def _cb(it, ms, fit, mode_ms, nm, user):
            ph = self.phase_times()
            r = IterReport(it, ms, fit, [mode_ms[i] for i in range(nm)],
                           ph if ph.size else None)
            reports.append(r)
            if callback is not None:
                callback(r)

        cb = N.ITER_CB(_cb)
        self._check(self._lib.cptc_als(self._h, int(iters), cb, None), "als")
        return reports
