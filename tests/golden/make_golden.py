#!/usr/bin/env python
"""Generates the golden fixtures of tests/golden/ by running the reference
program itself: zhixianzhu/cpTC's sources rebuilt for sm_100a by
oracle/build_ref.sh (oracle/_ref/cptc_opt), on a B200.

For each case the tensor comes from this repository's seeded generator, is
written as .tns, and cptc_opt runs with the case's switches.  Recorded: the
per-iteration fits it prints ("[ALS] iter ... fit=" / "[GEN] iter ... fit="),
the selector line, the final lambda and, where the reference can export
them, the final factors (ALS_EXPORT_FACTORS, %.20lf; GEN_DUMP, 17 digits).

  python tests/golden/make_golden.py [--out tests/golden]
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import cptc_b200 as cp  # noqa: E402

CASES = [
    # name, cfg, scale, iters, R, threshold, env
    ("cfg1_R16_fp64", 1, 1.0, 10, 16, 0.03, {"ALS_FORCE_CUDA": "1"}),
    ("cfg1_R16_tf32", 1, 1.0, 10, 16, 0.03, {"ALS_FORCE_WMMA": "1"}),
    ("cfg1_R32_auto", 1, 1.0, 5, 32, 0.03, {}),
    ("cfg4s_R32_fp64", 4, 0.002, 5, 32, 0.03, {"ALS_FORCE_CUDA": "1"}),
    ("cfg1_R8_generic", 1, 0.25, 5, 8, 0.03, {"ALS_GENERIC_FORCE": "1"}),
    ("cfg5s_R16_nodense", 5, 0.02, 5, 16, 0.03, {"GEN_DENSE": "0"}),
    ("cfg5s_R16_dense", 5, 0.02, 5, 16, 0.03, {"GEN_DENSE_THRESHOLD": "0.03"}),
    ("cfg5s_R8_pinv", 5, 0.01, 4, 8, 0.03, {"GEN_DENSE": "0", "GEN_SOLVER": "svd"}),
]


def parse(out: str) -> dict:
    fits, times = [], []
    for ln in out.splitlines():
        m = re.match(r"\[(ALS|GEN)\] iter (\d+)/(\d+) time=([\d.eE+-]+) ms.*fit=([-\d.eE+naif]+)", ln)
        if m:
            times.append(float(m.group(4)))
            fits.append(float(m.group(5)))
    lam = None
    for ln in out.splitlines():
        if ln.startswith("[ALS] Lambda:") or ln.startswith("[GEN] lambda ="):
            lam = [float(x) for x in ln.split(":" if "Lambda:" in ln else "=")[1].split()]
    sel = [ln for ln in out.splitlines() if "avg_fill=" in ln or "dense:" in ln or "reorder=" in ln]
    return {"fits": fits, "times_ms": times, "lambda": lam, "notes": sel}


def read_export(prefix: str, dims, R: int):
    F = []
    for n in range(len(dims)):
        p = Path(f"{prefix}.{n}.out")
        if not p.exists():
            return None
        vals = np.array([float(x) for x in p.read_text().split()[4:]])
        F.append(vals.reshape(dims[n], R))
    return F


def read_dump(path: str):
    lines = Path(path).read_text().splitlines()
    F, i = [], 0
    while i < len(lines):
        if lines[i].startswith("mode "):
            _, _, d, R = lines[i].split()
            rows = [list(map(float, lines[i + 1 + k].split())) for k in range(int(d))]
            F.append(np.array(rows))
            i += 1 + int(d)
        else:
            i += 1
    return F


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden"))
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    binary = ROOT / "oracle" / "_ref" / "cptc_opt"
    assert binary.exists(), "build the reference first (oracle/build_ref.sh)"
    out_dir = Path(a.out)
    out_dir.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory() as d:
        # the reference's own known-answer test (src/generic.cu:1389-1637)
        r = subprocess.run([str(binary)], env=dict(os.environ, GEN_SELFTEST="1"),
                           capture_output=True, text=True, timeout=600)
        (out_dir / "selftest.txt").write_text(r.stdout)
        for name, cfg, scale, iters, R, thr, env in CASES:
            if a.only and a.only not in name:
                continue
            t = cp.gen_config(cfg, scale)
            # the reference sizes each mode as max index + 1 (src/tensor.cu:247-254)
            t = cp.CooTensor(tuple(int(i.max()) + 1 for i in t.idx), t.idx, t.vals)
            tns = Path(d) / f"{name}.tns"
            cp.write_tns(tns, t)
            e = dict(os.environ, **env)
            exp = str(Path(d) / name)
            e["ALS_EXPORT_FACTORS"] = exp
            e["GEN_DUMP"] = exp
            r = subprocess.run([str(binary), str(tns), str(iters), str(R), str(thr)], env=e,
                               capture_output=True, text=True, timeout=1800)
            rec = {"case": name, "cfg": cfg, "scale": scale, "iters": iters, "R": R,
                   "threshold": thr, "env": env, "returncode": r.returncode,
                   "dims": list(t.dims), "nnz": t.nnz}
            rec.update(parse(r.stdout))
            F = read_export(exp, t.dims, R) if t.order == 3 and "ALS_GENERIC_FORCE" not in env \
                else (read_dump(exp + ".factors.txt") if Path(exp + ".factors.txt").exists()
                      else None)
            if F is not None:
                np.savez_compressed(out_dir / f"{name}_factors.npz", *F)
                rec["factors_file"] = f"{name}_factors.npz"
                rec["factor_space"] = "original" if "ALS_GENERIC_FORCE" not in env and \
                    t.order == 3 else "relabelled"
            (out_dir / f"{name}.json").write_text(json.dumps(rec, indent=1))
            print(name, r.returncode, rec["fits"][-3:] if rec["fits"] else r.stderr[-300:])


if __name__ == "__main__":
    main()
