"""cptc_residual_noalloc: the residual entry point that allocates nothing.

It keeps its per-block partial sums in one fixed array inside the library,
shared by every call, so the GPU test makes two calls in a row on different
tensors (the second with fewer nonzeros, so fewer partials) and checks each
against the allocating entry point cptc_residual on the same model, within
the FP64 bound the other parity tests use.  The file sorts last so that it
also runs after everything else has used the library in the same process.
"""
import ctypes as C

import numpy as np
import pytest

import cptc_b200 as cp
from cptc_b200 import _native as N

FP64_TOL = 1e-12


def _ptrs(xs):
    return (C.c_void_p * len(xs))(*[C.c_void_p(x) for x in xs])


def test_noalloc_rejects_sizes_beyond_its_limits():
    lib = N.engine_lib()
    dummy = _ptrs([0] * 8)
    for order, R in ((3, 129), (3, 0), (9, 16), (0, 16)):
        rc = lib.cptc_residual_noalloc(order, 10, dummy, None, R, dummy, None, None, None)
        assert rc == -4  # CPTC_E_UNSUP, raised before any CUDA call
        msg = lib.cptc_host_last_error().decode()
        assert "cptc_residual_noalloc" in msg and ("R must be" in msg or "order must be" in msg)


def _model(t, R, iters):
    """Engine state after `iters` ALS sweeps: the allocating residual, and
    the factors and lambda in the tensor's own labels."""
    e = cp.Engine(0)
    e.load(t)
    e.build(R, path="fp64")
    e.init_factors()
    e.als(iters)
    want = e.residual()["res_sq"]
    return want, e.factors(), e.lam(), e


def _noalloc(t, R, factors, lam):
    import torch

    dev = torch.device("cuda:0")
    idx = [torch.from_numpy(np.ascontiguousarray(i).view(np.int32)).to(dev) for i in t.idx]
    vals = torch.from_numpy(np.ascontiguousarray(t.vals)).to(dev)
    F = [torch.from_numpy(np.ascontiguousarray(f)).to(dev) for f in factors]
    lmb = torch.from_numpy(np.ascontiguousarray(lam)).to(dev)
    out = torch.full((1,), float("nan"), dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream(dev)
    lib = N.engine_lib()
    rc = lib.cptc_residual_noalloc(len(t.idx), int(t.vals.size), _ptrs([i.data_ptr() for i in idx]),
                                   vals.data_ptr(), int(R), _ptrs([f.data_ptr() for f in F]),
                                   lmb.data_ptr(), out.data_ptr(), C.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.cptc_host_last_error().decode()
    stream.synchronize()
    return float(out.item())


@pytest.mark.gpu
def test_noalloc_matches_allocating_residual_on_two_calls():
    cases = [
        # first call: many nonzeros -> every one of the 2048 partial slots in use
        (cp.gen_uniform((300, 250, 200), 900_000, seed=11, values="lognormal"), 24, 2),
        # second call: few nonzeros and another order -> far fewer partials;
        # slots the first call left behind must not leak into the sum
        (cp.gen_uniform((40, 30, 20, 10), 3_000, seed=12, values="normal"), 8, 1),
    ]
    for t, R, iters in cases:
        want, factors, lam, e = _model(t, R, iters)
        got = _noalloc(t, R, factors, lam)
        assert np.isfinite(got)
        assert abs(got - want) <= FP64_TOL * abs(want), (got, want)
        # anchored on the host as well: sum over the stored nonzeros of
        # (v - xhat)^2 in numpy, the bound test_exact_residual uses
        xhat = np.ones((t.nnz, R)) * lam
        for m in range(len(t.idx)):
            xhat = xhat * factors[m][t.idx[m]]
        host = float(np.sum((t.vals - xhat.sum(axis=1)) ** 2))
        assert abs(got - host) <= 1e-10 * host, (got, host)
        del e
