"""The CPU oracle against independent numpy restatements (no GPU)."""
import numpy as np
import pytest

import cptc_b200 as cp


def np_mttkrp(t, F, n):
    R = F[0].shape[1]
    out = np.zeros((t.dims[n], R))
    prod = np.repeat(t.vals[:, None], R, axis=1)
    for m in range(t.order):
        if m != n:
            prod = prod * F[m][t.idx[m]]
    np.add.at(out, t.idx[n], prod)
    return out


def rand_factors(dims, R, seed=1):
    rng = np.random.default_rng(seed)
    return [rng.random((d, R)) for d in dims]


@pytest.mark.parametrize("dims,nnz,R", [((30, 20, 40), 3000, 8), ((17, 33, 9, 12), 2500, 5),
                                        ((5, 7, 6, 4, 3), 400, 16), ((64, 1), 50, 3),
                                        ((5, 4, 3, 6, 4, 3), 600, 4),
                                        ((3, 2, 3, 2, 3, 2, 3, 2), 300, 2)])
def test_mttkrp_matches_numpy(oracle, dims, nnz, R):
    t = cp.gen_uniform(dims, nnz, seed=3, values="normal")
    F = rand_factors(t.dims, R)
    for n in range(t.order):
        ref = np_mttkrp(t, F, n)
        got = oracle.mttkrp(t, F, n, threads=2)
        assert np.allclose(got, ref, rtol=1e-13, atol=1e-13)


def test_mttkrp_threads_bitwise(oracle):
    t = cp.gen_uniform((40, 50, 60), 20000, seed=5)
    F = rand_factors(t.dims, 16)
    a = oracle.mttkrp(t, F, 1, threads=1)
    b = oracle.mttkrp(t, F, 1, threads=4)
    assert np.array_equal(a, b)


def test_hybrid_tf32_within_tolerance(oracle):
    # Dense 16^3 tiles (fill ~0.9) go through the TF32 slab arithmetic; the
    # reference's bound for that path is 2e-3 relative per entry.
    t = cp.gen_config(2, scale=0.02)
    F = rand_factors(t.dims, 32)
    for n in range(3):
        ref = oracle.mttkrp(t, F, n, threads=4)
        hyb, ntiles = oracle.mttkrp_hybrid3(t, F, n, thr=0.001, threads=4)
        assert ntiles > 0
        rel = np.abs(hyb - ref).max() / np.abs(ref).max()
        assert rel < 2e-3
        assert rel > 0  # the TF32 path really ran


def test_partition_stats(oracle):
    t = cp.gen_config(1)
    s = oracle.partition_stats3(t, thr=0.03)
    assert s["cutoff"] == 122
    assert s["dense_nnz"] + s["sparse_nnz"] == t.nnz
    # 200K over 512 tiles: every tile is dense (~390 nnz each)
    assert s["tiles"] == 512 and abs(s["avg_fill"] - t.nnz / (512 * 4096)) < 1e-12
    auto = oracle.partition_stats3(t, thr=0.0)
    assert 1 <= auto["cutoff"] <= 4096


def test_cadr_perm_is_degree_sorted(oracle):
    t = cp.gen_config(4, scale=0.001)
    for m in range(3):
        p = oracle.cadr_perm(t.dims[m], t.idx[m])
        assert sorted(p.tolist()) == list(range(t.dims[m]))
        deg = np.bincount(t.idx[m], minlength=t.dims[m])
        new_deg = np.empty_like(deg)
        new_deg[p] = deg
        assert np.all(np.diff(new_deg) <= 0)


def test_init_factors_uniform(oracle):
    F = oracle.init_factors3((10, 20, 30), 4)
    assert [f.shape for f in F] == [(10, 4), (20, 4), (30, 4)]
    allv = np.concatenate([f.ravel() for f in F])
    assert allv.min() >= 0.0 and allv.max() < 1.0
    # libstdc++: uniform_real_distribution<double> over mt19937(42) draws
    # two 32-bit words per double (generate_canonical<double, 53>).
    w0, w1 = 1608637542, 3421126067  # first two outputs of mt19937(42)
    assert F[0][0, 0] == (w0 + w1 * 2.0**32) / 2.0**64


def np_als3(t, R, iters):
    """numpy restatement of the order-3 ALS (src/als.cu:612-715) on factors
    from the oracle's init in CADR space (src/main.cu:178-219)."""
    from oracle import oracle as o
    perm = [o.cadr_perm(t.dims[m], t.idx[m]) for m in range(3)]
    idx = [perm[m][t.idx[m]] for m in range(3)]
    tt = cp.CooTensor(t.dims, [i.astype(np.uint32) for i in idx], t.vals)
    F = o.init_factors3(t.dims, R)
    lam = np.ones(R)
    X2 = float(t.vals @ t.vals)
    fits = []
    for _ in range(iters):
        for n in range(3):
            p, q = [m for m in range(3) if m != n]
            FtF = (F[p].T @ F[p]) * (F[q].T @ F[q])
            M = np_mttkrp(tt, F, n)
            w, V = np.linalg.eigh(FtF)
            tol = R * np.spacing(np.abs(w).max())
            keep = np.abs(w) > tol
            A = (V[:, keep] / w[keep]) @ V[:, keep].T
            Fn = M @ A.T / lam
            nr = np.linalg.norm(Fn, axis=0)
            Fn = np.where(nr < 1e-14, 0.0, Fn / np.where(nr < 1e-14, 1.0, nr))
            lam = np.where(nr < 1e-14, 0.0, lam * nr)
            F[n] = Fn
        G = [f.T @ f for f in F]
        iprod = float(lam @ np.einsum("kr,kr->r", F[2], M))
        model2 = float(lam @ (G[0] * G[1] * G[2]) @ lam)
        fits.append(1 - np.sqrt(max(X2 - 2 * iprod + model2, 0.0)) / np.sqrt(X2))
    return np.array(fits)


def test_als3_matches_numpy_restatement(oracle):
    t = cp.gen_uniform((20, 30, 25), 2500, seed=11, values="lognormal")
    fits, lam, F = oracle.cp_als3(t, 6, 6, path="fp64", threads=2, want_factors=True)
    ref = np_als3(t, 6, 6)
    assert np.max(np.abs(fits - ref)) < 1e-9
    assert np.all(np.diff(fits) > -1e-9)


def test_als3_planted_model_fit(oracle):
    # Sparse CP-ALS treats unobserved cells as zeros: on a 10% sample of a
    # rank-8 model the best fit is ~ sqrt(density)-limited, about 0.05.
    t = cp.gen_config(1)
    fits, lam, F = oracle.cp_als3(t, 16, 10, path="fp64", threads=4, want_factors=True)
    assert np.all(np.isfinite(fits)) and 0.03 < fits[-1] < 0.2
    assert np.all(np.diff(fits) > -1e-9)
    for f in F:
        nz = np.linalg.norm(f, axis=0)
        assert np.allclose(nz[lam > 0], 1.0, atol=1e-10)


def test_als3_tf32_close_to_fp64(oracle):
    t = cp.gen_config(1)
    f64, _, _ = oracle.cp_als3(t, 16, 5, path="fp64", threads=4)
    f32, _, _ = oracle.cp_als3(t, 16, 5, path="tf32", threads=4)
    assert np.max(np.abs(f64 - f32)) < 1e-3


def test_generic_als(oracle):
    t = cp.gen_config(5, scale=0.01)
    fits, lam, F = oracle.cp_als_generic(t, 8, 5, dense_thr=0.0, threads=4, want_factors=True)
    assert np.all(np.isfinite(fits)) and fits[-1] > 0.0
    fits2, _, _ = oracle.cp_als_generic(t, 8, 5, dense_thr=0.0, reorder="none", threads=4)
    # relabelling carries the initial rows along, so the model is unchanged
    assert np.max(np.abs(fits - fits2)) < 1e-9


def test_generic_units_close_to_fp64(oracle):
    t = cp.gen_config(5, scale=0.05)
    f64, _, _ = oracle.cp_als_generic(t, 16, 3, dense_thr=0.0, threads=4)
    f32, _, _ = oracle.cp_als_generic(t, 16, 3, dense_thr=0.03, threads=4)
    assert np.max(np.abs(f64 - f32)) < 1e-3


def test_hits_reorder_permutation(oracle):
    t = cp.gen_config(5, scale=0.01)
    ranks = oracle.reorder(t, "hits", rounds=3)
    for m, r in enumerate(ranks):
        assert sorted(r.tolist()) == list(range(t.dims[m]))
