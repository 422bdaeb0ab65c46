"""The multi-GPU partition and collectives on CPU ranks (gloo), no GPU needed.

tests/multirank.py restates the engine's distributed ALS (rows in slabs of
equal nonzero weight with each rank keeping its rows' nonzeros, a heavy prefix
of rows shared out by nonzero and all-reduced, one exchange per mode: Gram
all-reduce, heavy-row all-reduce and the slabs in one all-reduce) over world-size 2 and 3
gloo groups; it must reproduce the single-process ALS, and every rank must end
with the same factors.  One tensor has a head row larger than a rank's share,
so that row is split between ranks.
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
            rank, fits, F, lam, shares, heavy = q.get(timeout=240)
            out[rank] = (fits, F, lam, shares, heavy)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(out[r][0], str), out[r][0]
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_als_matches_single_process(world):
    spec = dict(dims=(90, 70, 50), nnz=12_000, seed=21, values="lognormal", R=8, iters=4)
    out = _run(world, spec)
    t = make_cpu_case(spec)
    ref = np_als3(t, spec["R"], spec["iters"])
    fits0, F0, lam0, shares0, heavy0 = out[0]
    assert np.max(np.abs(fits0 - ref)) < 1e-10
    for r in range(1, world):
        fits, F, lam, shares, heavy = out[r]
        assert np.array_equal(fits, fits0) and np.array_equal(lam, lam0)
        for a, b in zip(F, F0):
            assert np.array_equal(a, b)
    # every nonzero is on exactly one rank for every target mode
    for m in range(3):
        assert sum(out[r][3][m] for r in range(world)) == spec["nnz"]


def test_sharded_als_with_a_split_head_row():
    # 45% of the nonzeros in row 0 of every mode (like config 4's head
    # block): the first block is the heavy prefix, its nonzeros are dealt to
    # the 3 ranks and its partial rows all-reduced; the rest is balanced
    spec = dict(dims=(60, 50, 40), nnz=9_000, seed=5, values="lognormal", R=8, iters=3,
                heavy=0.45)
    t = make_cpu_case(spec)
    assert np.bincount(t.idx[0]).max() / t.nnz > 1 / 3
    out = _run(3, spec)
    ref = np_als3(t, spec["R"], spec["iters"])
    assert np.max(np.abs(out[0][0] - ref)) < 1e-10
    for a, b in zip(out[2][1], out[0][1]):
        assert np.array_equal(a, b)
    assert all(h >= 16 for h in out[0][4])  # a heavy prefix in every mode
    for m in range(3):
        sizes = [out[r][3][m] for r in range(3)]
        assert sum(sizes) == spec["nnz"]
        assert max(sizes) < 0.45 * spec["nnz"]  # the head row no longer sits on one rank


def test_sharded_als_with_every_row_in_the_heavy_prefix():
    # few 16-row blocks, each above an eighth of a rank's share on 4 ranks:
    # every row of every mode is in the heavy prefix, so no rank owns a slab
    # and each mode update is the prefix's all-reduce alone
    spec = dict(dims=(80, 64, 12), nnz=6_000, seed=9, values="lognormal", R=8, iters=3)
    out = _run(4, spec)
    assert list(out[0][4]) == list(spec["dims"])
    t = make_cpu_case(spec)
    ref = np_als3(t, spec["R"], spec["iters"])
    assert np.max(np.abs(out[0][0] - ref)) < 1e-10
    for r in range(1, 4):
        assert np.array_equal(out[r][0], out[0][0])
        for a, b in zip(out[r][1], out[0][1]):
            assert np.array_equal(a, b)
    for m in range(3):
        assert sum(out[r][3][m] for r in range(4)) == spec["nnz"]
