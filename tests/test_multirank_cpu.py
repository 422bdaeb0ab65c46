"""The multi-GPU partition and collectives on CPU ranks (gloo), no GPU needed.

tests/multirank.py restates the engine's distributed ALS (nonzeros shared out
by count, partial MTTKRP reduce-scattered into equal row slabs, Gram
all-reduce, slab all-gather; or the peer exchange's rank-order sums) over
world-size 2 and 3 gloo groups; it must reproduce the single-process ALS, and
every rank must end with the same factors.  The tensor has a Zipf-like head row so that one row is split
between ranks.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest

import cptc_b200 as cp

from multirank import cpu_worker, make_cpu_case
from test_oracle import np_als3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, spec):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=cpu_worker, args=(r, world, port, spec, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, fits, F, lam, shares = q.get(timeout=240)
            out[rank] = (fits, F, lam, shares)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(out[r][0], str), out[r][0]
    return out


@pytest.mark.parametrize("world,exchange", [(2, "nccl"), (3, "nccl"), (3, "peer")])
def test_sharded_als_matches_single_process(world, exchange):
    spec = dict(dims=(90, 70, 50), nnz=12_000, seed=21, values="lognormal", R=8, iters=4,
                exchange=exchange)
    out = _run(world, spec)
    t = make_cpu_case(spec)
    ref = np_als3(t, spec["R"], spec["iters"])
    fits0, F0, lam0, shares0 = out[0]
    assert np.max(np.abs(fits0 - ref)) < 1e-10
    for r in range(1, world):
        fits, F, lam, shares = out[r]
        assert np.array_equal(fits, fits0) and np.array_equal(lam, lam0)
        for a, b in zip(F, F0):
            assert np.array_equal(a, b)
    # nonzeros are shared out by count: shares differ by at most one
    for m in range(3):
        sizes = [out[r][3][m] for r in range(world)]
        assert sum(sizes) == spec["nnz"] and max(sizes) - min(sizes) <= 1


def test_peer_exchange_sums_in_rank_order():
    # the peer exchange adds the ranks' partials in rank order on every rank:
    # the replicas agree bit for bit, and with the NCCL sums to rounding
    spec = dict(dims=(60, 50, 40), nnz=9_000, seed=5, values="lognormal", R=8, iters=3,
                heavy=0.45, exchange="peer")
    out = _run(3, spec)
    ref = _run(3, dict(spec, exchange="nccl"))
    for r in (1, 2):
        assert np.array_equal(out[r][0], out[0][0])
        for a, b in zip(out[r][1], out[0][1]):
            assert np.array_equal(a, b)
    assert np.max(np.abs(out[0][0] - ref[0][0])) < 1e-12


def test_sharded_als_with_a_split_head_row():
    # 45% of the nonzeros in row 0 of every mode (like config 4's head block):
    # with 3 ranks that row is computed in pieces by two ranks and summed by
    # the reduce-scatter
    spec = dict(dims=(60, 50, 40), nnz=9_000, seed=5, values="lognormal", R=8, iters=3,
                heavy=0.45)
    t = make_cpu_case(spec)
    assert np.bincount(t.idx[0]).max() / t.nnz > 1 / 3
    out = _run(3, spec)
    ref = np_als3(t, spec["R"], spec["iters"])
    assert np.max(np.abs(out[0][0] - ref)) < 1e-10
    for a, b in zip(out[2][1], out[0][1]):
        assert np.array_equal(a, b)
