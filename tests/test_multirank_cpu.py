"""The multi-GPU row-slab path on CPU ranks (gloo), no GPU needed.

The slab cuts come from cptc_slab_cuts, the host function the engine uses to
partition each mode; the distributed ALS restatement in tests/multirank.py
runs the engine's sequence of collectives (partial-Gram all-reduce, one
broadcast per slab owner, dot-product all-reduce) over world-size 2 and 3
gloo groups and must reproduce the single-process ALS.
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest

import cptc_b200 as cp

from multirank import cpu_worker
from test_oracle import np_als3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_slab_cuts_properties():
    rng = np.random.default_rng(3)
    for dim, world in ((1000, 2), (1000, 8), (37, 4), (5, 3), (16, 2), (300, 7)):
        counts = rng.zipf(1.3, dim).astype(np.uint32) % 5000
        nnz = int(counts.sum())
        cuts = cp.slab_cuts(counts, nnz, world).astype(np.int64)
        assert cuts[0] == 0 and cuts[-1] == dim and len(cuts) == world + 1
        assert np.all(np.diff(cuts) >= 0)
        inner = cuts[1:-1]
        assert np.all((inner % 16 == 0) | (inner == dim))
        # rank r starts at the first 16-row boundary at or after the row where
        # the running count reaches r/world of nnz
        csum = np.concatenate([[0], np.cumsum(counts, dtype=np.int64)])
        for r in range(1, world):
            row = int(np.argmax(csum[1:] * world >= r * nnz))
            want = min(-(-(row + 1) // 16) * 16, dim)
            assert cuts[r] == max(want, cuts[r - 1])


def test_slab_cuts_rejects_bad_arguments():
    with pytest.raises(ValueError):
        cp.slab_cuts(np.ones(4, np.uint32), 4, 0)


def test_mode_slabs_balance_uniform_tensor():
    t = cp.gen_uniform((512, 640, 384), 200_000, seed=5)
    for world in (2, 4, 8):
        for m, cuts in enumerate(cp.mode_slabs(t, world)):
            share = [np.count_nonzero((t.idx[m] >= a) & (t.idx[m] < b))
                     for a, b in zip(cuts[:-1], cuts[1:])]
            assert sum(share) == t.nnz
            # each slab is within one 16-row block of its equal share
            per_row = t.nnz / t.dims[m]
            assert max(share) <= t.nnz / world + 32 * per_row


@pytest.mark.parametrize("world", [2, 3])
def test_slab_als_matches_single_process(world):
    spec = dict(dims=(90, 70, 50), nnz=12_000, seed=21, values="lognormal", R=8, iters=4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=cpu_worker, args=(r, world, port, spec, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, fits, F, lam, cuts = q.get(timeout=240)
            out[rank] = (fits, F, lam, cuts)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert not isinstance(out[r][0], str), out[r][0]
    t = cp.gen_uniform(spec["dims"], spec["nnz"], seed=spec["seed"], values=spec["values"])
    ref = np_als3(t, spec["R"], spec["iters"])
    fits0, F0, lam0, cuts0 = out[0]
    assert np.max(np.abs(fits0 - ref)) < 1e-10
    # every slab is non-trivial and every rank ends with identical factors
    assert all(len(set(c)) == world + 1 for c in cuts0)
    for r in range(1, world):
        fits, F, lam, _ = out[r]
        assert np.array_equal(fits, fits0) and np.array_equal(lam, lam0)
        for a, b in zip(F, F0):
            assert np.array_equal(a, b)
