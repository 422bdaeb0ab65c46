"""CUDA engine (through the C ABI) against the CPU oracle on identical inputs.

Tolerances are the reference's own bounds: FP64 paths 1e-12 relative
(atomic reordering only), the TF32 dense-tile path 2e-3 relative per entry,
and final fit 1e-4 absolute.  Norm-wise relative error is used for the FP64
MTTKRP: || got - ref || / || ref ||.
"""
import os

import numpy as np
import pytest

import cptc_b200 as cp

pytestmark = pytest.mark.gpu

FP64_TOL = 1e-12


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def rand_factors(dims, R, seed=7, signed=False):
    rng = np.random.default_rng(seed)
    return [(rng.standard_normal((d, R)) if signed else rng.random((d, R))) for d in dims]


def engine_for(t, R, **kw):
    e = cp.Engine(0)
    e.load(t)
    e.build(R, **kw)
    return e


CASES = [
    # dims, nnz, R, values
    ((128, 128, 128), 200000, 16, "uniform"),
    ((128, 128, 128), 200000, 8, "normal"),
    ((37, 45, 29), 5000, 17, "normal"),
    ((37, 45, 29), 5000, 32, "lognormal"),
    ((3000, 20, 50), 60000, 64, "uniform"),  # mode-1 rows of ~3000 nnz span tasks
    ((500, 400, 300), 30000, 128, "normal"),
    ((200, 1, 300), 4000, 24, "uniform"),    # a mode of length 1
    ((60, 50, 40), 8000, 1, "normal"),        # rank 1
]


@pytest.mark.parametrize("dims,nnz,R,values", CASES)
def test_mttkrp_fp64_order3(gpu, oracle, dims, nnz, R, values):
    t = cp.gen_uniform(dims, nnz, seed=21, values=values)
    e = engine_for(t, R, path="fp64")
    F = rand_factors(t.dims, R, signed=(values == "normal"))
    for m in range(3):
        e.set_factor(m, F[m])
    for n in range(3):
        got = e.mttkrp(n)
        ref = oracle.mttkrp(t, F, n, threads=8)
        assert rel(got, ref) < FP64_TOL, (n, rel(got, ref))


def test_mttkrp_empty_rows_and_heavy_row(gpu, oracle):
    # Indices only in the lower half of each mode, plus one row holding
    # ~40% of the nonzeros: empty rows must come out exactly zero and the
    # heavy row is split over many tasks (atomic combination).
    rng = np.random.default_rng(3)
    n = 50000
    i = rng.integers(0, 60, n)
    i[: n * 2 // 5] = 7
    j = rng.integers(0, 50, n)
    k = rng.integers(0, 40, n)
    key = np.unique((i * 1000 + j) * 1000 + k)
    t = cp.CooTensor((120, 100, 80), [(key // 1000000).astype(np.uint32),
                                       (key // 1000 % 1000).astype(np.uint32),
                                       (key % 1000).astype(np.uint32)],
                     rng.standard_normal(len(key)))
    R = 32
    e = engine_for(t, R, path="fp64")
    F = rand_factors(t.dims, R, signed=True)
    for m in range(3):
        e.set_factor(m, F[m])
    for mode in range(3):
        got = e.mttkrp(mode)
        ref = oracle.mttkrp(t, F, mode, threads=8)
        assert rel(got, ref) < FP64_TOL
        empty = np.setdiff1d(np.arange(t.dims[mode]), t.idx[mode])
        assert np.all(got[empty] == 0.0)


@pytest.mark.parametrize("order,R", [(4, 8), (4, 128), (5, 64), (6, 8), (6, 32), (6, 128)])
def test_mttkrp_fp64_nway_records(gpu, oracle, order, R):
    # orders 4-6 at the ranks with 32-byte records (o3 is used at order 6),
    # every mode as the target, against the oracle's COO MTTKRP
    dims = (17, 23, 11, 29, 13, 19)[:order]
    t = cp.gen_uniform(dims, 12_000, seed=40 + order, values="normal")
    e = engine_for(t, R, dense_generic=False, reorder="none")
    F = rand_factors(t.dims, R, signed=True)
    for m in range(order):
        e.set_factor(m, F[m])
    for n in range(order):
        ref = oracle.mttkrp(t, F, n, threads=8)
        assert rel(e.mttkrp(n), ref) < FP64_TOL, (order, R, n)


@pytest.mark.parametrize("dims,nnz,R", [((30, 20, 25, 40), 20000, 16),
                                        ((12, 9, 15, 8, 11), 8000, 32),
                                        ((300, 200), 5000, 8),
                                        ((9, 7, 8, 6, 7, 5, 6), 9000, 16),      # order 7
                                        ((6, 5, 7, 4, 6, 5, 4, 6), 9000, 8)])  # order 8
def test_mttkrp_fp64_generic(gpu, oracle, dims, nnz, R):
    t = cp.gen_uniform(dims, nnz, seed=5, values="normal")
    e = engine_for(t, R, dense_generic=False)
    F = rand_factors(t.dims, R, signed=True)
    for m in range(t.order):
        e.set_factor(m, F[m])
    for n in range(t.order):
        assert rel(e.mttkrp(n), oracle.mttkrp(t, F, n, threads=8)) < FP64_TOL


@pytest.mark.parametrize("R", [16, 32, 64, 128])
def test_mttkrp_tf32_tiles(gpu, oracle, R):
    # config 2's 256^3 layout at 5% of its nonzeros, every tile taken as
    # dense (threshold 0.001); partition on the given coordinates (no
    # relabelling) so both sides see the same tiles.
    t = cp.gen_config(2, scale=0.05)
    e = engine_for(t, R, path="tf32", threshold=0.001, reorder="none")
    st = e.stats()
    assert st["tf32_path"] == 1 and st["dense_tiles"] > 0
    F = rand_factors(t.dims, R)
    for m in range(3):
        e.set_factor(m, F[m])
    for n in range(3):
        got = e.mttkrp(n)
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.001, threads=8)
        exact = oracle.mttkrp(t, F, n, threads=8)
        assert rel(got, hyb) < 1e-5
        assert np.abs(got - exact).max() / np.abs(exact).max() < 2e-3


@pytest.mark.parametrize("R", [16, 32, 128])
def test_mttkrp_tf32_full_tiles(gpu, oracle, R):
    # 64^3 at fill ~0.9: 64 tiles of ~3,700 nonzeros each, more than the
    # tile kernel stages in shared memory ahead of time (the rest of each
    # tile is read directly)
    t = cp.gen_uniform((64, 64, 64), 235_000, seed=8, values="lognormal")
    e = engine_for(t, R, path="tf32", threshold=0.03, reorder="none")
    st = e.stats()
    assert st["tf32_path"] == 1 and st["dense_tiles"] == 64
    assert st["dense_nnz"] / st["dense_tiles"] > 2048
    F = rand_factors(t.dims, R)
    for m in range(3):
        e.set_factor(m, F[m])
    for n in range(3):
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.03, threads=8)
        assert rel(e.mttkrp(n), hyb) < 1e-5


@pytest.mark.parametrize("R", [8, 32])
def test_mttkrp_tf32_ragged_dims(gpu, oracle, R):
    # dims that are not multiples of 16: the last tile block of every mode
    # is partial, so the kernel's row guards decide which rows exist
    # (the reference's GEN_SELFTEST covers the same edge, src/generic.cu:1420-1426)
    t = cp.gen_uniform((50, 37, 45), 40_000, seed=14, values="lognormal")
    e = engine_for(t, R, path="tf32", threshold=0.01, reorder="none")
    st = e.stats()
    assert st["tf32_path"] == 1 and st["dense_tiles"] == 4 * 3 * 3
    F = rand_factors(t.dims, R)
    for m in range(3):
        e.set_factor(m, F[m])
    for n in range(3):
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.01, threads=8)
        assert rel(e.mttkrp(n), hyb) < 1e-5


def test_mttkrp_tf32_mixed_partition(gpu, oracle):
    t = cp.gen_config(3, scale=0.02)
    e = engine_for(t, 32, path="tf32", threshold=0.03, reorder="none")
    st = e.stats()
    ref_stats = oracle.partition_stats3(t, thr=0.03)
    assert st["dense_tiles"] == ref_stats["tiles"]
    assert st["dense_nnz"] == ref_stats["dense_nnz"]
    assert st["cutoff"] == ref_stats["cutoff"]
    F = rand_factors(t.dims, 32)
    for m in range(3):
        e.set_factor(m, F[m])
    for n in range(3):
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.03, threads=8)
        assert rel(e.mttkrp(n), hyb) < 1e-5


def test_als3_fp64_matches_oracle(gpu, oracle):
    t = cp.gen_config(1)
    e = engine_for(t, 16, path="fp64")
    e.init_factors()
    rep = e.als(10)
    fits = np.array([r.fit for r in rep])
    ref, lam_ref, F_ref = oracle.cp_als3(t, 16, 10, path="fp64", threads=8, want_factors=True)
    assert np.max(np.abs(fits - ref)) < 1e-8
    lam = e.lam()
    assert np.allclose(np.sort(lam), np.sort(lam_ref), rtol=1e-6)
    for m in range(3):
        assert rel(e.factor(m), F_ref[m]) < 1e-6


def test_als3_tf32_close_to_oracle(gpu, oracle):
    t = cp.gen_config(1)
    e = engine_for(t, 16, path="tf32")
    e.init_factors()
    fits = np.array([r.fit for r in e.als(5)])
    ref_tf32, _, _ = oracle.cp_als3(t, 16, 5, path="tf32", threads=8)
    ref_fp64, _, _ = oracle.cp_als3(t, 16, 5, path="fp64", threads=8)
    assert np.max(np.abs(fits - ref_tf32)) < 1e-5
    assert np.max(np.abs(fits - ref_fp64)) < 1e-4


def test_als_generic_matches_oracle(gpu, oracle):
    t = cp.gen_config(5, scale=0.02)
    e = engine_for(t, 16, dense_generic=False)
    e.init_factors()
    fits = np.array([r.fit for r in e.als(5)])
    ref, _, _ = oracle.cp_als_generic(t, 16, 5, dense_thr=0.0, threads=8)
    assert np.max(np.abs(fits - ref)) < 1e-8


def test_als_generic_pinv_solver(gpu, oracle):
    t = cp.gen_uniform((40, 30, 20, 10), 8000, seed=2, values="poisson")
    e = engine_for(t, 8, dense_generic=False, solver="pinv")
    e.init_factors()
    fits = np.array([r.fit for r in e.als(4)])
    ref, _, _ = oracle.cp_als_generic(t, 8, 4, dense_thr=0.0, solver="pinv", threads=8)
    assert np.max(np.abs(fits - ref)) < 1e-8


def test_order3_generic_route(gpu, oracle):
    # ALS_GENERIC_FORCE: order 3 through the N-order path (CADR with tie
    # break, Cholesky, lambda = norms).
    t = cp.gen_config(1, scale=0.2)
    e = engine_for(t, 8, generic=True)
    e.init_factors()
    fits = np.array([r.fit for r in e.als(4)])
    ref, _, _ = oracle.cp_als_generic(t, 8, 4, dense_thr=0.0, threads=8)
    assert np.max(np.abs(fits - ref)) < 1e-8


@pytest.mark.parametrize("R,inner", [(16, (0, 1, 2)), (32, (0, 1, 2)), (16, (1, 2, 3)),
                                     (8, (0, 2, 3))])
def test_mttkrp_units_generic(gpu, oracle, R, inner):
    # N-order dense units (16^3 over the inner modes, outer modes fixed) in
    # TF32 with FP64 weighting, plus the FP64 residual; no relabelling so
    # both sides form the same units.  Inner sets other than (0,1,2) are
    # refused by the reference (its kernel fails its own self-test there).
    t = cp.gen_config(5, scale=0.05)
    thr = 0.03 if inner == (0, 1, 2) else 0.002  # other inner sets form fewer full units
    e = engine_for(t, R, reorder="none", dense_thr_generic=thr, dense_inner=inner)
    st = e.stats()
    assert st["tf32_path"] == 1 and st["dense_tiles"] > 0
    F = rand_factors(t.dims, R)
    for m in range(t.order):
        e.set_factor(m, F[m])
    for n in range(t.order):
        got = e.mttkrp(n)
        exact = oracle.mttkrp(t, F, n, threads=8)
        if n in inner:
            ref = units_oracle(oracle, t, F, inner, inner.index(n), thr)
            assert rel(got, ref) < 1e-5
            assert np.abs(got - exact).max() / np.abs(exact).max() < 2e-3
        else:
            assert rel(got, exact) < FP64_TOL


import ctypes as _C  # noqa: E402


def units_oracle(oracle, t, F, inner, tslot, thr):
    a = oracle._Args(t)
    Fs, fp = oracle._fptrs(F)
    out = np.zeros((t.dims[inner[tslot]], F[0].shape[1]))
    inn = (_C.c_int * 3)(*inner)
    oracle.lib().or_mttkrp_units(t.order, a.dims, a.nnz, a.ip, a.vp, F[0].shape[1], fp, inn,
                                 tslot, thr, out.ctypes.data_as(oracle.DP), 8)
    return out


@pytest.mark.parametrize("order", [3, 4])
def test_exact_residual(gpu, order):
    # cptc_residual: sum over the stored nonzeros of (v - xhat)^2 with the
    # current factors and lambda, against numpy in the caller's labels
    dims = (60, 50, 40) if order == 3 else (30, 20, 25, 15)
    t = cp.gen_uniform(dims, 20_000, seed=31, values="lognormal")
    e = engine_for(t, 16, path="fp64")
    e.init_factors()
    e.als(2)
    F, lam = e.factors(), e.lam()
    xhat = np.ones((t.nnz, 16)) * lam
    for m in range(t.order):
        xhat = xhat * F[m][t.idx[m]]
    want = float(np.sum((t.vals - xhat.sum(axis=1)) ** 2))
    got = e.residual()
    assert abs(got["res_sq"] - want) <= 1e-10 * want
    assert abs(got["x_sq"] - float(t.vals @ t.vals)) <= 1e-12 * got["x_sq"]


def test_phase_times(gpu):
    # the phase events change no result; phase 0 is the MTTKRP time the
    # iteration callback reports, and the phases fit inside the iteration
    t = cp.gen_config(1)
    runs = []
    for on in (False, True):
        e = engine_for(t, 16)
        e.init_factors()
        if on:
            e.set_phase_timing(True)
        runs.append(e.als(4))
        if on:
            ph = e.phase_times()
            assert ph.shape == (3, len(cp.Engine.PHASES))
            e.set_phase_timing(False)
            assert e.als(1)[0].phases is None and e.phase_times().size == 0
        e.close()
    off, on = runs
    # FP64 atomics order the MTTKRP sums differently from run to run (~1e-16)
    # and the ALS iterations amplify that (measured: 2e-12 after 4 of them)
    assert np.max(np.abs(np.subtract([r.fit for r in off], [r.fit for r in on]))) < 1e-9
    for r in on:
        assert r.phases.shape == (3, 5) and np.all(r.phases >= 0)
        assert np.allclose(r.phases[:, 0], r.mode_ms)
        assert r.phases.sum() <= r.ms + 1e-3
    assert all(r.phases is None for r in off)


def test_sharded_factor_upload_on_one_gpu(gpu):
    # one rank: the sharded upload is the plain upload (relabelled or not)
    t = cp.gen_config(1, scale=0.2)
    for reorder in ("default", "none"):
        e = engine_for(t, 8, path="fp64", reorder=reorder)
        F = rand_factors(t.dims, 8, signed=True)
        for m in range(3):
            e.set_factor(m, F[m], sharded=True)
        for m in range(3):
            assert np.array_equal(e.factor(m), F[m])
            assert np.array_equal(e.factor(m, sharded=True), F[m])
        e.close()


def _block(rng, lo, ext, fill):
    """Distinct cells of the box [lo, lo + ext) at the given fill."""
    cells = np.array(np.meshgrid(*[np.arange(l, l + e) for l, e in zip(lo, ext)],
                                 indexing="ij")).reshape(len(lo), -1).T
    return cells[rng.random(len(cells)) < fill]


def _distinct(dims, parts, rng, values="lognormal"):
    c = np.unique(np.concatenate(parts).astype(np.uint64) @ np.array(
        [np.prod(dims[m + 1:], dtype=np.uint64) for m in range(len(dims))], dtype=np.uint64))
    idx, rest = [], c
    for m in range(len(dims) - 1, -1, -1):
        idx.append((rest % np.uint64(dims[m])).astype(np.uint32))
        rest = rest // np.uint64(dims[m])
    idx = idx[::-1]
    v = rng.lognormal(0.0, 1.0, len(c)) if values == "lognormal" else rng.standard_normal(len(c))
    return cp.CooTensor(tuple(dims), idx, v)


@pytest.mark.parametrize("path", ["fp64", "tf32"])
def test_mttkrp_modes_beyond_32768(gpu, oracle, path):
    # Mode lengths 70000 and 40000 (the reference packs coordinates into 15-bit
    # fields and drops the residual beyond 32767, src/partition.cu:1896-1906):
    # a uniform residual plus dense blocks at coordinates >= 32768, one of
    # them the partial last block of mode 1 (300 = 18*16 + 12)
    rng = np.random.default_rng(31)
    dims = (70000, 300, 40000)
    parts = [np.stack([rng.integers(0, d, 150_000) for d in dims], axis=1),
             _block(rng, (69984, 288, 39984), (16, 12, 16), 0.6),
             _block(rng, (32768, 0, 32768), (16, 16, 16), 0.5),
             _block(rng, (40000, 100, 16), (32, 16, 16), 0.4)]
    t = _distinct(dims, parts, rng)
    R = 32
    e = engine_for(t, R, path=path, threshold=0.03, reorder="none")
    F = rand_factors(t.dims, R)
    for m in range(3):
        e.set_factor(m, F[m])
    if path == "tf32":
        st = e.stats()
        ps = oracle.partition_stats3(t, thr=0.03)
        assert st["tf32_path"] == 1 and st["dense_tiles"] == ps["tiles"] == 6
        assert st["dense_nnz"] == ps["dense_nnz"]
    for n in range(3):
        got = e.mttkrp(n)
        exact = oracle.mttkrp(t, F, n, threads=8)
        if path == "fp64":
            assert rel(got, exact) < FP64_TOL, n
        else:
            hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.03, threads=8)
            assert rel(got, hyb) < 1e-5, n
            nz = exact != 0.0
            assert np.max(np.abs(got - exact)[nz] / np.abs(exact)[nz]) < 2e-3, n


@pytest.mark.parametrize("dense", [False, True])
def test_mttkrp_order4_mode_beyond_32768(gpu, oracle, dense):
    # order 4 with a 40000-row mode, FP64 records, and dense units over the
    # inner modes (0, 1, 2) with a block at rows >= 32768
    rng = np.random.default_rng(32)
    dims = (40000, 30, 20, 25)
    parts = [np.stack([rng.integers(0, d, 80_000) for d in dims], axis=1)]
    for l in range(3):
        b = _block(rng, (36000, 0, 0), (16, 16, 16), 0.5)
        parts.append(np.concatenate([b, np.full((len(b), 1), l)], axis=1))
    t = _distinct(dims, parts, rng)
    R = 16
    e = engine_for(t, R, dense_generic=dense, reorder="none")
    assert e.stats()["tf32_path"] == (1 if dense else 0)
    F = rand_factors(t.dims, R)
    for m in range(4):
        e.set_factor(m, F[m])
    for n in range(4):
        got = e.mttkrp(n)
        exact = oracle.mttkrp(t, F, n, threads=8)
        if not dense:
            assert rel(got, exact) < FP64_TOL, n
        else:
            nz = exact != 0.0
            assert np.max(np.abs(got - exact)[nz] / np.abs(exact)[nz]) < 2e-3, n


def test_mttkrp_full_size_config4_entrywise(gpu, oracle):
    # Config 4 at full size (76.9M nonzeros), R=32, hybrid path, mode 2: every
    # entry against the oracle's TF32 emulation (1e-5 norm-wise) and against
    # the exact FP64 MTTKRP (2e-3 per entry).  The tensor is relabelled with
    # the oracle's restatement of the reference's CADR, so the partition is
    # the reference's (81,886 tiles, 37,821,322 residual nonzeros).
    t = cp.gen_config(4)
    dims = tuple(int(i.max()) + 1 for i in t.idx)
    idx = []
    for m in range(3):
        perm = oracle.cadr_perm(dims[m], t.idx[m]).astype(np.uint32)
        idx.append(perm[t.idx[m]])
    u = cp.CooTensor(dims, idx, t.vals)
    R = 32
    e = engine_for(u, R, path="tf32", threshold=0.03, reorder="none")
    st = e.stats()
    assert st["dense_tiles"] == 81886 and st["sparse_nnz"] == 37821322
    F = rand_factors(u.dims, R, seed=9)
    for m in range(3):
        e.set_factor(m, F[m])
    got = e.mttkrp(2)
    e.close()
    threads = os.cpu_count() or 8
    hyb, _ = oracle.mttkrp_hybrid3(u, F, 2, thr=0.03, threads=threads)
    assert rel(got, hyb) < 1e-5
    exact = oracle.mttkrp(u, F, 2, threads=threads)
    nz = exact != 0.0
    assert np.max(np.abs(got - exact)[nz] / np.abs(exact)[nz]) < 2e-3
    assert np.all(got[~nz] == 0.0)


@pytest.mark.parametrize("kind,sample", [("hits", 8_000_000), ("hits", 250_000), ("cadr", 0)])
def test_device_relabelling_matches_oracle(gpu, oracle, kind, sample):
    # Config 5 at full size (3.3M nonzeros, order 4): HITS scores summed on
    # the device in the reference's order give the same ranks, bit for bit,
    # as the oracle's sequential restatement (src/generic.cu:1290-1341), with
    # the whole tensor as the sample and with a strided sample; the degree
    # order breaks ties by index
    t = cp.gen_config(5)
    t = cp.CooTensor(tuple(int(i.max()) + 1 for i in t.idx), t.idx, t.vals)
    e = cp.Engine(0)
    e.load(t)
    e.build(16, generic=True, reorder=kind, reorder_rounds=3, reorder_sample=max(sample, 1),
            dense_generic=False)
    ref = oracle.reorder(t, kind, rounds=3, sample=max(sample, 1))
    for m in range(t.order):
        assert np.array_equal(e.relabel(m), ref[m]), m
    assert e.stats()["reorder_ms"] > 0.0
    e.close()
