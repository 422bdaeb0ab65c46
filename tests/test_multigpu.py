"""The engine's sharded row-slab ALS on 2 GPUs against the same engine on 1 GPU.

Each case runs tests/multirank.py under torchrun (one process per GPU; gloo
only to pass the NCCL unique id) and compares rank 0's fits, lambda, factors
and a final MTTKRP with a single-GPU run of the same build.  Sums are the same
terms in another order, so FP64 agrees to rounding; the TF32 tiles compute
each tile identically on either layout.  Every rank's replica must hold the
same bits.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import cptc_b200 as cp

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("case", ["fp64_o3", "hybrid_o3", "hybrid_o3_r128", "generic_o4",
                                  "fp64_o3_r17"])
def test_two_gpu_slab_als_matches_one_gpu(case, tmp_path):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    from multirank import GPU_CASES, make_case

    out = tmp_path / f"{case}.npz"
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(HERE.parent), str(HERE)]),
               **GPU_CASES[case].get("env", {}))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(HERE / "multirank.py"), "--out", str(out),
           "--case", case]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.load(out)

    spec = GPU_CASES[case]
    t = make_case(spec)
    e = cp.Engine(0)
    e.load(t)
    e.build(spec["R"], **spec["build"])
    e.init_factors()
    fits = np.array([x.fit for x in e.als(spec["iters"])])
    F = e.factors()
    lam = e.lam()
    M0 = e.mttkrp(0)
    st = e.stats()
    e.close()

    assert int(got["tf32"]) == int(st["tf32_path"])
    assert int(got["replicas_equal"]) == 1
    assert int(got["sharded_ok"]) == 1
    tol = 1e-6 if st["tf32_path"] else 1e-9
    assert np.max(np.abs(got["fits"] - fits)) < tol * 10
    assert rel(got["lam"], lam) < tol
    for m, f in enumerate(F):
        assert rel(got[f"F{m}"], f) < tol, m
    assert rel(got["M0"], M0) < tol
