"""Worker code for the multi-rank tests (imported by spawned processes).

`shard_als3` restates, with numpy on CPU ranks, what the engine does on G GPUs
for the order-3 ALS (cptc_b200/csrc/cuda/shard.cu, comm.cu):
  * rows of each mode are cut into 16-row blocks; a block's weight is its
    nonzero count; the heavy prefix ends with the last block above an eighth
    of a rank's share, and the remaining blocks are cut into G contiguous
    slabs of equal weight (each cut at the nearest block boundary);
  * each rank keeps the nonzeros of its slab and, of the heavy prefix's
    nonzeros (in the tensor's order), every G-th one starting at its rank;
  * per mode: local MTTKRP -> solve of the own slab rows -> one all-reduce
    of [the heavy rows' partial MTTKRP | every rank's solved slab rows,
    zeros elsewhere | Gram partial and fit dots] -> every rank solves the
    heavy rows itself and adds their Gram and dots -> every rank normalises
    the whole factor.
Run with gloo it checks the partition and the payload of the collectives on
the host.
"""
from __future__ import annotations

import datetime
import hashlib
import os
import sys

import numpy as np


def np_mttkrp(idx, vals, dims, F, n):
    R = F[0].shape[1]
    out = np.zeros((dims[n], R))
    prod = np.repeat(vals[:, None], R, axis=1)
    for m in range(len(dims)):
        if m != n:
            prod = prod * F[m][idx[m]]
    np.add.at(out, idx[n], prod)
    return out


def truncated_pinv(A, R):
    w, V = np.linalg.eigh(A)
    tol = R * np.spacing(np.abs(w).max())
    keep = np.abs(w) > tol
    return (V[:, keep] / w[keep]) @ V[:, keep].T


MAX_HEAVY_ROWS = 4096


def shard_plan(rows_idx, dim, world):
    """(heavy rows, row cut points, block cut points) of one mode from the
    target indices of its nonzeros (every nonzero weighs 1)."""
    nb = -(-dim // 16)
    w = np.bincount(rows_idx // 16, minlength=nb).astype(np.float64)
    W = w.sum()
    heavy = np.nonzero(w > W / (8.0 * world))[0]
    h = int(heavy[-1]) + 1 if heavy.size else 0
    h = min(h, MAX_HEAVY_ROWS // 16)
    Wn = w[h:].sum()
    cb = [h] + [nb] * world
    acc, b = 0.0, h
    for r in range(1, world):
        target = Wn * r / world
        while b < nb and acc + 0.5 * w[b] <= target:
            acc += w[b]
            b += 1
        cb[r] = b
    slab = [0] + [min(c * 16, dim) for c in cb[1:world]] + [dim]
    return min(h * 16, dim), slab, cb


def shard_select(rows_idx, H, cb, rank, world):
    """Positions of this rank's nonzeros for one target mode."""
    blk = rows_idx // 16
    hb = -(-H // 16)
    heavy = blk < hb
    hord = np.cumsum(heavy) - heavy  # ordinal among the heavy nonzeros
    mine = np.where(heavy, hord % world == rank, (blk >= cb[rank]) & (blk < cb[rank + 1]))
    return np.nonzero(mine)[0]


def shard_als3(t, R, iters, rank, world, dist):
    """The engine's distributed order-3 ALS on `world` CPU ranks (see module doc)."""
    import torch

    from oracle import oracle as o

    perm = [o.cadr_perm(t.dims[m], t.idx[m]) for m in range(3)]
    idx = [perm[m][t.idx[m]].astype(np.int64) for m in range(3)]
    F = [f.copy() for f in o.init_factors3(t.dims, R)]
    lam = np.ones(R)
    G = [f.T @ f for f in F]
    X2 = float(t.vals @ t.vals)
    fits = []
    plan = [shard_plan(idx[n], t.dims[n], world) for n in range(3)]
    mine = [shard_select(idx[n], plan[n][0], plan[n][2], rank, world) for n in range(3)]

    def allreduce(x):
        v = torch.from_numpy(np.ascontiguousarray(x))
        dist.all_reduce(v)
        return v.numpy()

    def exchange(M, Fn, hdr, n):
        # one all-reduce over [MTTKRP rows of the heavy prefix | this rank's
        # solved rows past it, zeros elsewhere | Gram and dot partials]
        # (comm.cu: comm_exchange_mode)
        H, slab, _ = plan[n]
        lo, hi = max(slab[rank], H), max(slab[rank + 1], H)
        buf = np.zeros((t.dims[n], R))
        buf[:H] = M[:H]
        buf[lo:hi] = Fn[lo:hi]
        red = allreduce(np.concatenate([buf.ravel(), hdr]))
        rows = red[:t.dims[n] * R].reshape(t.dims[n], R)
        M[:H] = rows[:H]
        Fn[H:] = rows[H:]
        return red[t.dims[n] * R:]

    for _ in range(iters):
        for n in range(3):
            p, q = [m for m in range(3) if m != n]
            A = truncated_pinv(G[p] * G[q], R)
            H, slab, _ = plan[n]
            lo, hi = max(slab[rank], H), max(slab[rank + 1], H)
            sel = mine[n]
            M = np_mttkrp([i[sel] for i in idx], t.vals[sel], t.dims, F, n)
            Fn = np.zeros((t.dims[n], R))
            Fn[lo:hi] = M[lo:hi] @ A.T / lam
            payload = [(Fn[lo:hi].T @ Fn[lo:hi]).ravel()]
            if n == 2:
                payload.append(np.einsum("kr,kr->r", Fn[lo:hi], M[lo:hi]))
            red = exchange(M, Fn, np.concatenate(payload), n)
            if H > 0:  # the heavy rows, solved by every rank, added once
                Fn[:H] = M[:H] @ A.T / lam
                red[:R * R] += (Fn[:H].T @ Fn[:H]).ravel()
                if n == 2:
                    red[R * R:] += np.einsum("kr,kr->r", Fn[:H], M[:H])
            Gs = red[:R * R].reshape(R, R)
            nr = np.sqrt(np.diag(Gs))
            zero = nr < 1e-14
            scale = np.where(zero, 0.0, 1.0 / np.where(zero, 1.0, nr))
            lam = np.where(zero, 0.0, lam * nr)
            F[n] = Fn * scale
            G[n] = Gs * np.outer(scale, scale)
        dots = red[R * R:] * scale
        iprod = float(lam @ dots)
        model2 = float(lam @ (G[0] * G[1] * G[2]) @ lam)
        fits.append(1 - np.sqrt(max(X2 - 2 * iprod + model2, 0.0)) / np.sqrt(X2))
    return np.array(fits), F, lam, [int(m.size) for m in mine], [pl[0] for pl in plan]


def make_cpu_case(spec):
    """Seeded tensor of a CPU test; spec["heavy"] = f moves the first f of the
    nonzeros into row 0 of every mode (a head row larger than a rank's share)."""
    import cptc_b200 as cp

    t = cp.gen_uniform(spec["dims"], spec["nnz"], seed=spec["seed"], values=spec["values"])
    k = int(spec.get("heavy", 0.0) * t.nnz)
    for m in range(t.order):
        t.idx[m][:k] = 0
    return t


def cpu_worker(rank, world, port, spec, q):
    """Entry point of one spawned gloo rank: runs shard_als3 and reports."""
    import torch.distributed as dist

    import cptc_b200 as cp

    os.environ.setdefault("OMP_NUM_THREADS", "1")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        t = make_cpu_case(spec)
        fits, F, lam, shares, heavy = shard_als3(t, spec["R"], spec["iters"], rank, world, dist)
        q.put((rank, fits, F, lam, shares, heavy))
    except Exception as e:  # report instead of hanging the other ranks' test
        q.put((rank, repr(e), None, None, None, None))
        raise
    finally:
        dist.destroy_process_group()


def gpu_main(argv=None):
    """One torchrun rank of the engine's NCCL row-slab ALS; rank 0 writes
    fits, lambda and factors (original labels) to --out as .npz."""
    import argparse

    import torch
    import torch.distributed as dist

    import cptc_b200 as cp

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--case", required=True)
    a = ap.parse_args(argv)
    spec = GPU_CASES[a.case]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        t = make_case(spec)
        e = cp.Engine(local)
        obj = [cp.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        e.comm_init(obj[0], rank, world)
        e.load(t)
        e.build(spec["R"], **spec["build"])
        e.init_factors()
        reps = e.als(spec["iters"])
        st = e.stats()
        F = e.factors()
        lam = e.lam()
        M0 = e.mttkrp(0)
        # sharded upload: each rank's host copy holds only its own rows (NaN
        # elsewhere); every replica must end with all of them
        s_ok = True
        for m in range(t.order):
            full = F[m] * 0.5 + 0.25
            rows = -(-full.shape[0] // world)
            part = np.full_like(full, np.nan)
            part[rank * rows:(rank + 1) * rows] = full[rank * rows:(rank + 1) * rows]
            e.set_factor(m, part, sharded=True)
            s_ok &= bool(np.array_equal(e.factor(m), full))
            back = np.full_like(full, np.nan)
            e.factor(m, out=back, sharded=True)  # only this rank's rows written
            s_ok &= bool(np.array_equal(back, part, equal_nan=True))
        for m in range(t.order):  # back to the ALS result
            e.set_factor(m, F[m])
        # every rank's replica must hold the same bits
        h = hashlib.sha1(b"".join(np.ascontiguousarray(f).tobytes() for f in F)).hexdigest()
        hashes = [None] * world
        dist.all_gather_object(hashes, h)
        dist.barrier()
        if rank == 0:
            np.savez(a.out, fits=np.array([r.fit for r in reps]), lam=lam, M0=M0,
                     tf32=int(st["tf32_path"]), replicas_equal=int(len(set(hashes)) == 1),
                     sharded_ok=int(s_ok),
                     **{f"F{m}": f for m, f in enumerate(F)})
        e.close()
    finally:
        dist.destroy_process_group()


GPU_CASES = {
    "fp64_o3": dict(gen=("uniform", (600, 500, 400), 400_000, 3, "lognormal"), R=16, iters=4,
                    build=dict(path="fp64")),
    "hybrid_o3": dict(gen=("config", 4, 0.05, 0), R=32, iters=3, build=dict(path="tf32")),
    "hybrid_o3_r128": dict(gen=("config", 4, 0.02, 0), R=128, iters=2, build=dict(path="tf32")),
    "generic_o4": dict(gen=("config", 5, 0.2, 0), R=16, iters=3, build=dict(generic=True)),
    # R=17: odd rank on the FP64 path
    "fp64_o3_r17": dict(gen=("uniform", (301, 250, 199), 60_000, 4, "normal"), R=17, iters=3,
                        build=dict(path="fp64")),
}


def make_case(spec):
    import cptc_b200 as cp

    g = spec["gen"]
    if g[0] == "uniform":
        return cp.gen_uniform(g[1], g[2], seed=g[3], values=g[4])
    return cp.gen_config(g[1], scale=g[2], seed=g[3])


if __name__ == "__main__":
    gpu_main()
