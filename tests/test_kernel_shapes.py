"""The kernel shapes and launch orders selectable for measurement
(CPTC_REC3_R32=8x4, CPTC_REC3_R128=u2, CPTC_TILES_SHAPE=nw2,
CPTC_OVERLAP_TILES=1) compute what the defaults do.

The library reads these switches once per process, so each shape runs in a
child process (this file's __main__) that writes its MTTKRPs to a .npz; the
test compares them with the CPU oracle: FP64 to 1e-12, TF32 tiles to 1e-5
against the oracle's TF32 emulation.
"""
import argparse
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def case_tensor(kind):
    import cptc_b200 as cp

    if kind == "zipf":  # config 4's index distribution, 0.5% of its nonzeros
        t = cp.gen_config(4, scale=0.005)
        return cp.CooTensor(tuple(int(i.max()) + 1 for i in t.idx), t.idx, t.vals)
    if kind == "mixed":  # config 3 at 2%: dense tiles and a residual
        return cp.gen_config(3, scale=0.02)
    return cp.gen_uniform((64, 64, 64), 120_000, seed=8, values="lognormal")


def factors(dims, R):
    rng = np.random.default_rng(11)
    return [rng.standard_normal((d, R)) for d in dims]


def worker(kind, R, path, out):
    import cptc_b200 as cp

    t = case_tensor(kind)
    e = cp.Engine(0)
    e.load(t)
    e.build(R, path=path, threshold=0.03, reorder="none")
    F = factors(t.dims, R)
    for m in range(3):
        e.set_factor(m, F[m])
    np.savez(out, tf32=int(e.stats()["tf32_path"]), **{f"M{n}": e.mttkrp(n) for n in range(3)})
    e.close()


def run_shape(env_extra, kind, R, path, tmp_path):
    out = tmp_path / "m.npz"
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(HERE.parent), str(HERE)]),
               **env_extra)
    r = subprocess.run([sys.executable, str(Path(__file__)), "--kind", kind, "--R", str(R),
                        "--path", path, "--out", str(out)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return np.load(out)


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("env,R", [({"CPTC_REC3_R32": "8x4"}, 32),
                                   ({"CPTC_REC3_R128": "u2"}, 128)])
def test_residual_shapes(gpu, oracle, env, R, tmp_path):
    got = run_shape(env, "zipf", R, "fp64", tmp_path)
    t = case_tensor("zipf")
    F = factors(t.dims, R)
    for n in range(3):
        assert rel(got[f"M{n}"], oracle.mttkrp(t, F, n, threads=8)) < 1e-12, n


@pytest.mark.parametrize("R", [16, 32, 128])
def test_tile_shape_nw2(gpu, oracle, R, tmp_path):
    got = run_shape({"CPTC_TILES_SHAPE": "nw2"}, "dense", R, "tf32", tmp_path)
    assert int(got["tf32"]) == 1
    t = case_tensor("dense")
    F = factors(t.dims, R)
    for n in range(3):
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.03, threads=8)
        assert rel(got[f"M{n}"], hyb) < 1e-5, n


@pytest.mark.parametrize("R", [32, 128])
def test_tiles_beside_residual(gpu, oracle, R, tmp_path):
    # CPTC_OVERLAP_TILES=1: the tile kernel on its own stream into a second
    # buffer, added after both kernels
    got = run_shape({"CPTC_OVERLAP_TILES": "1"}, "mixed", R, "tf32", tmp_path)
    assert int(got["tf32"]) == 1
    t = case_tensor("mixed")
    F = factors(t.dims, R)
    for n in range(3):
        hyb, _ = oracle.mttkrp_hybrid3(t, F, n, thr=0.03, threads=8)
        assert rel(got[f"M{n}"], hyb) < 1e-5, n


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--kind", required=True)
    ap.add_argument("--R", type=int, required=True)
    ap.add_argument("--path", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    worker(a.kind, a.R, a.path, a.out)
