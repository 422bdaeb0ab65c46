"""Every launch shape of the order-3 dense-tile kernel against the oracle.

The tile kernel picks its shape from R: n-tiles per warp (1, 2, 3 or 4),
words staged per tile (1024, or 512 above R=64) and resident CTAs per SM
(5, 4 or 3).  Each shape runs on tiles below and above its stage size (the
rest of a large tile is read from global memory), with partial blocks at
the end of every mode, and is compared with the oracle's TF32 emulation
(1e-5 norm-wise) and the exact FP64 MTTKRP (2e-3 per entry).
"""
import numpy as np
import pytest

import cptc_b200 as cp

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("R", [8, 16, 24, 32, 40, 64, 72, 128])
@pytest.mark.parametrize("fill", ["sparse", "full"])
def test_tile_kernel_shapes(gpu, oracle, R, fill):
    if fill == "sparse":  # ~300-700 nonzeros per tile, ragged dims
        t = cp.gen_uniform((50, 37, 45), 40_000, seed=14, values="lognormal")
    else:  # ~3,700 nonzeros per tile: above both stage sizes
        t = cp.gen_uniform((48, 48, 40), 78_000, seed=15, values="lognormal")
    e = cp.Engine(0)
    e.load(t)
    e.build(R, path="tf32", threshold=0.01, reorder="none")
    assert e.stats()["tf32_path"] == 1
    rng = np.random.default_rng(R)
    F = [rng.random((d, R)) for d in t.dims]
    for m in range(3):
        e.set_factor(m, F[m])
    for n in range(3):
        got = e.mttkrp(n)
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.01, threads=8)
        assert rel(got, hyb) < 1e-5, (R, fill, n)
        exact = oracle.mttkrp(t, F, n, threads=8)
        nz = exact != 0.0
        assert np.max(np.abs(got - exact)[nz] / np.abs(exact)[nz]) < 2e-3, (R, fill, n)
    e.close()
