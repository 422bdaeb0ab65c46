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
