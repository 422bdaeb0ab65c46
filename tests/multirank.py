"""Worker code for the multi-rank tests (imported by spawned processes).

`shard_als3` restates, with numpy on CPU ranks, what the engine does on G GPUs
for the order-3 ALS.  Work and ownership are split separately:
  * work: the nonzeros of each mode, sorted by target row, are cut into G
    equal-count chunks (the engine gives each rank an equal range of its
    nonzero-balanced tasks and an equal-weight range of the dense tiles), so
    a heavy row is shared by several ranks;
  * ownership: rows in G equal slabs (ceil(I/G) rows each).
Per mode: partial MTTKRP of the rank's chunk -> reduce-scatter into the slabs
-> solve of the own slab -> one all-reduce of the partial Gram (column norms
are its diagonal; the last mode appends the fit's column dot products) beside
the all-gather of the unnormalised slabs -> every rank normalises the whole
factor.  Run with gloo it checks the order and payload of the collectives on
the host.  exchange="peer" restates the peer-memory exchange instead: every
rank's partial slab rows reach the owner (region r of its receive buffer) and
the owner adds the G partials in rank order 0..G-1; the Gram partials go to
slot r of every rank, which adds the slots in rank order.
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


def shard_als3(t, R, iters, rank, world, dist, exchange="nccl"):
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
    srows = [-(-d // world) for d in t.dims]
    # this rank's nonzeros per target mode: an equal share of the row-sorted order
    chunk = []
    for n in range(3):
        order = np.argsort(idx[n], kind="stable")
        a, b = t.nnz * rank // world, t.nnz * (rank + 1) // world
        chunk.append(order[a:b])

    def allreduce(x):
        v = torch.from_numpy(np.ascontiguousarray(x))
        dist.all_reduce(v)
        return v.numpy()

    def gather(x):
        parts = [torch.zeros(x.shape, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(x)))
        return [p.numpy() for p in parts]

    def rank_order_sum(parts):
        acc = np.zeros_like(parts[0])
        for p in parts:  # r = 0 .. world-1
            acc = acc + p
        return acc

    def reduce_scatter_rows(M, s, n):
        # padded to world * s rows; gloo has no reduce_scatter: all-reduce, keep own slab
        P = np.zeros((world * s, R))
        P[:M.shape[0]] = M
        if exchange == "peer":
            # region r of the owner's receive buffer holds rank r's rows of its
            # slab, pushed only inside rank r's touched rows [lo_r, hi_r)
            rows = idx[n][chunk[n]]
            hull = np.array([rows.min(), rows.max() + 1] if rows.size else [0, 0])
            hulls = gather(hull.astype(np.float64))
            parts = []
            for r, g in enumerate(gather(P)):
                reg = np.zeros((s, R))
                lo, hi = int(hulls[r][0]), int(hulls[r][1])
                a, b = max(lo, rank * s), min(hi, (rank + 1) * s)
                if r == rank:
                    reg = g[rank * s:(rank + 1) * s]
                elif a < b:
                    reg[a - rank * s:b - rank * s] = g[a:b]
                parts.append(reg)
            return rank_order_sum(parts)
        return allreduce(P)[rank * s:(rank + 1) * s]

    def reduce_slots(x):
        if exchange == "peer":
            return rank_order_sum(gather(x))
        return allreduce(x)

    def allgather_rows(Fl, s, dim):
        parts = [torch.zeros((s, R), dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(Fl)))
        return np.concatenate([p.numpy() for p in parts])[:dim]

    for _ in range(iters):
        for n in range(3):
            p, q = [m for m in range(3) if m != n]
            FtF = G[p] * G[q]
            mine = chunk[n]
            M = np_mttkrp([i[mine] for i in idx], t.vals[mine], t.dims, F, n)
            s = srows[n]
            lo, hi = min(rank * s, t.dims[n]), min((rank + 1) * s, t.dims[n])
            Ms = reduce_scatter_rows(M, s, n)       # own slab, padded to s rows
            A = truncated_pinv(FtF, R)
            Fl = np.zeros((s, R))
            Fl[:hi - lo] = Ms[:hi - lo] @ A.T / lam
            # one all-reduce (Gram partials, and for the last mode the fit's
            # column dots of the unnormalised rows) beside the all-gather of
            # the unnormalised slab; every rank then normalises the factor
            payload = [(Fl.T @ Fl).ravel()]
            if n == 2:
                payload.append(np.einsum("kr,kr->r", Fl[:hi - lo], Ms[:hi - lo]))
            red = reduce_slots(np.concatenate(payload))
            Gs = red[:R * R].reshape(R, R)
            Fn = allgather_rows(Fl, s, t.dims[n])
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
    return np.array(fits), F, lam, [c.size for c in chunk]


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
        fits, F, lam, shares = shard_als3(t, spec["R"], spec["iters"], rank, world, dist,
                                          spec.get("exchange", "nccl"))
        q.put((rank, fits, F, lam, shares))
    except Exception as e:  # report instead of hanging the other ranks' test
        q.put((rank, repr(e), None, None, None))
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
    "generic_o4": dict(gen=("config", 5, 0.2, 0), R=16, iters=3, build=dict(generic=True)),
}
# the same cases with the peer-memory exchange (a 1-GPU run ignores it)
for _k in list(GPU_CASES):
    GPU_CASES[_k + "_peer"] = dict(GPU_CASES[_k], build=dict(GPU_CASES[_k]["build"],
                                                             exchange="peer"))
# other rank cut points (the split changes only which rank sums which part)
GPU_CASES["fp64_o3_rowcost"] = dict(GPU_CASES["fp64_o3"], env={"CPTC_TASK_ROW_COST": "4"})
GPU_CASES["hybrid_o3_tilecost_peer"] = dict(GPU_CASES["hybrid_o3_peer"],
                                            env={"CPTC_TILE_FIXED_COST": "1200",
                                                 "CPTC_TASK_ROW_COST": "4"})
# R=17: odd slabs take the scalar copy kernels
GPU_CASES["fp64_o3_r17_peer"] = dict(gen=("uniform", (301, 250, 199), 60_000, 4, "normal"), R=17,
                                     iters=3, build=dict(path="fp64", exchange="peer"))


def peer_timeout_main(out: str):
    """Two torchrun ranks with the peer exchange and a 1 s barrier limit:
    rank 0 runs one ALS iteration alone, so its first barrier waits for a
    flag that nothing sets; the kernel gives up, the iteration fails with
    CPTC_E_COMM, and after a collective rebuild both ranks run ALS again."""
    import time

    import torch
    import torch.distributed as dist

    import cptc_b200 as cp

    os.environ["CPTC_PEER_TIMEOUT_MS"] = "1000"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        t = cp.gen_uniform((200, 150, 100), 20_000, seed=7, values="uniform")
        e = cp.Engine(local)
        obj = [cp.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        e.comm_init(obj[0], rank, world)
        e.load(t)
        e.build(8, path="fp64", exchange="peer")
        e.init_factors()
        e.als(1)
        dist.barrier()
        code, waited = 0, 0.0
        if rank == 0:
            t0 = time.perf_counter()
            try:
                e.als(1)
            except cp.CptcError as x:
                code = x.code
            waited = time.perf_counter() - t0
        dist.barrier()  # rank 1 waits here, off the GPU
        e.build(8, path="fp64", exchange="peer")
        e.init_factors()
        fits = [r.fit for r in e.als(3)]
        allf = [None] * world
        dist.all_gather_object(allf, fits)
        if rank == 0:
            np.savez(out, code=code, waited=waited, fits=np.array(fits),
                     ranks_agree=int(all(f == fits for f in allf)))
        e.close()
    finally:
        dist.destroy_process_group()


def comm_timeout_main(out: str):
    """Two torchrun ranks on the NCCL exchange with CPTC_COMM_TIMEOUT_MS=2000:
    rank 0 runs one ALS iteration alone, so its reduce-scatter waits for a
    rank that never joins; the host wait gives up, aborts the communicator
    and reports CPTC_E_COMM.  Both ranks then leave without touching the
    aborted communicator again."""
    import time

    import torch
    import torch.distributed as dist

    import cptc_b200 as cp

    os.environ["CPTC_COMM_TIMEOUT_MS"] = "2000"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    t = cp.gen_uniform((200, 150, 100), 20_000, seed=7, values="uniform")
    e = cp.Engine(local)
    obj = [cp.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    e.comm_init(obj[0], rank, world)
    e.load(t)
    e.build(8, path="fp64")
    e.init_factors()
    ok_fits = [r.fit for r in e.als(2)]
    dist.barrier()
    code, waited = 0, 0.0
    if rank == 0:
        t0 = time.perf_counter()
        try:
            e.als(1)
        except cp.CptcError as x:
            code = x.code
        waited = time.perf_counter() - t0
        np.savez(out, code=code, waited=waited, fits=np.array(ok_fits))
    dist.barrier()  # rank 1 waits here, off the GPU
    dist.destroy_process_group()
    # the peer of an aborted communicator may not be able to destroy its own
    # cleanly: leave without running the destructors
    sys.stdout.flush()
    os._exit(0)


def make_case(spec):
    import cptc_b200 as cp

    g = spec["gen"]
    if g[0] == "uniform":
        return cp.gen_uniform(g[1], g[2], seed=g[3], values=g[4])
    return cp.gen_config(g[1], scale=g[2], seed=g[3])


if __name__ == "__main__":
    if len(sys.argv) > 2 and sys.argv[1] == "--peer-timeout":
        peer_timeout_main(sys.argv[2])
    elif len(sys.argv) > 2 and sys.argv[1] == "--comm-timeout":
        comm_timeout_main(sys.argv[2])
    else:
        gpu_main()
