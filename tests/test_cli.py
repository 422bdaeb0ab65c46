"""The drop-in command-line driver (cptc_opt): reference argv, switches and
output lines, checked against the reference's own printed fits."""
import json
import os
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import cptc_b200 as cp

ROOT = Path(__file__).resolve().parent.parent
CLI = ROOT / "cptc_b200" / "_lib" / "cptc_opt"
GOLD = ROOT / "tests" / "golden"


def golden_tensor(g, path):
    t = cp.gen_config(g["cfg"], g["scale"])
    t = cp.CooTensor(tuple(int(i.max()) + 1 for i in t.idx), t.idx, t.vals)
    cp.write_tns(path, t)
    return t


def run(args, env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([str(CLI)] + [str(a) for a in args], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return r.stdout


def fits_of(out, tag):
    return np.array([float(m.group(1)) for m in
                     re.finditer(rf"\[{tag}\] iter \d+/\d+ time=[\d.eE+-]+ ms.*fit=([-\d.eE+]+)",
                                 out)])


def test_cli_binary_built():
    assert CLI.exists()


def test_cli_binary_cache_switch(tmp_path):
    # the load happens before the engine starts, so the cache lines show on
    # a machine without a GPU too (the run then stops at cptc_create)
    t = cp.gen_uniform((20, 30, 40), 500, seed=1)
    p = tmp_path / "c.tns"
    cp.write_tns(p, t)
    env = dict(os.environ, CPTC_TNS_CACHE="1")
    outs = [subprocess.run([str(CLI), str(p), "1", "8"], env=env, capture_output=True,
                           text=True, timeout=300).stdout for _ in range(2)]
    assert "[Main] binary cache: written from the text" in outs[0]
    assert "[Main] binary cache: read" in outs[1]
    assert "NNZ: 500" in outs[1]
    u, hit = cp.read_tns_cached(p)
    assert hit and np.array_equal(u.vals, t.vals)
    named = tmp_path / "named.bin"
    env["CPTC_TNS_CACHE"] = str(named)
    subprocess.run([str(CLI), str(p), "1", "8"], env=env, capture_output=True, timeout=300)
    assert named.exists()


@pytest.mark.gpu
def test_cli_order3_tf32_matches_reference(gpu, tmp_path):
    g = json.loads((GOLD / "cfg1_R32_auto.json").read_text())
    tns = tmp_path / "t.tns"
    t = golden_tensor(g, tns)
    exp = tmp_path / "exp"
    out = run([tns, g["iters"], g["R"], g["threshold"]],
              {"ALS_FORCE_WMMA": "1", "ALS_EXPORT_FACTORS": str(exp)})
    fits = fits_of(out, "ALS")
    assert len(fits) == g["iters"]
    assert np.max(np.abs(fits - np.array(g["fits"]))) < 1e-5
    assert "[ALS] Lambda:" in out and "[ALS] Final RMSE=" in out
    # the selector line up to the threshold is the reference's, character for
    # character (the threshold itself is this build's B200 rule)
    ref_sel = next(ln for ln in g["notes"] if "avg_fill=" in ln)
    sel = next(ln for ln in out.splitlines() if "avg_fill=" in ln)
    assert sel.split(" (")[0] == ref_sel.split(" (")[0]
    head = (tmp_path / "exp.0.out").read_text().split("\n")[:3]
    assert head == ["matrix", "2", f"{t.dims[0]} {g['R']}"]
    lam = (tmp_path / "exp.lambda.out").read_text().split()
    assert lam[:3] == ["vector", "1", str(g["R"])] and len(lam) == 3 + g["R"]


@pytest.mark.gpu
def test_cli_generic_matches_reference(gpu, tmp_path):
    g = json.loads((GOLD / "cfg5s_R16_dense.json").read_text())
    tns = tmp_path / "t.tns"
    golden_tensor(g, tns)
    out = run([tns, g["iters"], g["R"], g["threshold"]],
              {"GEN_DENSE_THRESHOLD": "0.03", "GEN_DUMP": str(tmp_path / "d")})
    fits = fits_of(out, "GEN")
    assert np.max(np.abs(fits - np.array(g["fits"]))) < 1e-5
    assert "[GEN] exact:" in out
    assert (tmp_path / "d.factors.txt").read_text().startswith("# cpTC factor dump")


def _gpu_count() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def test_cli_ranks_end_together_when_one_fails(tmp_path):
    # CPTC_NGPU=3 on a machine without GPUs: every rank fails at cptc_create;
    # the job must end (no rank left waiting for the others) with a failure
    # status, and only rank 0 prints
    if _gpu_count() > 0:
        pytest.skip("checks the failure path; needs a machine without GPUs")
    t = cp.gen_uniform((20, 30, 40), 500, seed=1)
    p = tmp_path / "t.tns"
    cp.write_tns(p, t)
    r = subprocess.run([str(CLI), str(p), "1", "8"], env=dict(os.environ, CPTC_NGPU="3"),
                       capture_output=True, text=True, timeout=120)
    assert r.returncode != 0
    assert r.stdout.count("[Main] Load time") == 1


@pytest.mark.gpu
def test_cli_two_gpus_match_one(gpu, tmp_path):
    # one process per GPU from the command line: the same fits as one GPU
    if _gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    g = json.loads((GOLD / "cfg1_R32_auto.json").read_text())
    tns = tmp_path / "t.tns"
    golden_tensor(g, tns)
    one = fits_of(run([tns, g["iters"], g["R"], g["threshold"]], {"ALS_FORCE_CUDA": "1"}), "ALS")
    two_out = run([tns, g["iters"], g["R"], g["threshold"]],
                  {"ALS_FORCE_CUDA": "1", "CPTC_NGPU": "2"})
    two = fits_of(two_out, "ALS")
    assert len(two) == len(one) == g["iters"]
    assert np.max(np.abs(two - one)) < 1e-8
    assert two_out.count("[ALS] Final RMSE=") == 1


def _selftest_counts(txt):
    """(inner set, pass) -> (units, dense_nnz) from GEN_SELFTEST output."""
    out, key = {}, None
    for ln in txt.splitlines():
        m = re.search(r"inner=\((\d),(\d),(\d)\) pass (\d)", ln)
        if m:
            key = (m.group(1) + m.group(2) + m.group(3), int(m.group(4)))
        m = re.search(r"units=(\d+) dense_nnz=(\d+)", ln)
        if m and key is not None:
            out[key] = (int(m.group(1)), int(m.group(2)))
    return out


@pytest.mark.gpu
def test_cli_selftest_known_answers(gpu):
    # GEN_SELFTEST=1: the reference's own known-answer test of the N-order
    # dense path on the same tensor (mt19937(1234); nnz 16827 as the
    # reference prints it).  Every inner-mode set passes here, including the
    # three the reference's kernel fails, with the reference's unit counts.
    r = subprocess.run([str(CLI)], env=dict(os.environ, GEN_SELFTEST="1"),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "[SELFTEST] N=4 dims=40,24,36,3 nnz=16827 R=8" in r.stdout
    assert "[SELFTEST] PASSED (0 failures)" in r.stdout
    assert r.stdout.count("OK") == 24
    ref = _selftest_counts((GOLD / "selftest.txt").read_text())
    got = _selftest_counts(r.stdout)
    assert set(got) == set(ref)
    assert got == ref


def test_cli_density_line_text():
    # the selector line keeps the reference's labels (src/main.cu:408-416),
    # which scripts grep for
    src = (ROOT / "cptc_b200" / "csrc" / "cli" / "cptc_opt.cpp").read_text()
    assert "[Main] 稠密度检测: dense_nnz=" in src
    assert "(阈值 %g) -> %s" in src
    assert "双流串行(WMMA+FP64)" in src and "纯 CUDA core(全 FP64)" in src
    for label in ("sparse_nnz=", "tiles=", "avg_fill=", "eff_dense=", "dense_ratio="):
        assert label in src


def test_generator_executable_matches_library(tmp_path):
    # cptc_gen writes the tensor cptc_gen_config makes (the reference arm of
    # bench.py feeds it to the reference's driver)
    gen = ROOT / "cptc_b200" / "_lib" / "cptc_gen"
    p = tmp_path / "g.tns"
    r = subprocess.run([str(gen), "3", "0.002", str(p)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    info = json.loads(r.stdout.strip().splitlines()[-1])
    t = cp.gen_config(3, 0.002)
    u = cp.read_tns(p)
    assert info["nnz"] == t.nnz == u.nnz and info["nominal_dims"] == list(t.dims)
    assert info["dims"] == list(u.dims)
    for m in range(3):
        assert np.array_equal(u.idx[m], t.idx[m])
    assert np.array_equal(u.vals, t.vals)
