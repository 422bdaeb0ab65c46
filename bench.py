#!/usr/bin/env python
"""CP-ALS benchmark: seconds per ALS iteration on the 76.9M-nonzero order-3
power-law tensor (config 4).

Workload: order-3 synthetic tensor 12092 x 9184 x 28818 with 76.9M nonzeros,
Zipf(1.1) indices per mode over a random permutation, lognormal values
(cptc_gen_config(4)); CP rank R=32 (R=128 with --rank 128, and an R=128
sub-record in every default run); one step = one CP-ALS iteration (3 mode
updates + Gram fit).  The tensor views are streamed from HBM every MTTKRP
(1.2 GB per mode, larger than the 126 MB L2), so no explicit L2 flush is
needed between steps.

  python bench.py [--gpus N --steps K --warmup W --rank R]
  python bench.py --impl reference ...   # cpTC's own build (oracle/_ref)

One JSON line on rank 0: metric, value, unit, e2e, roofline, cpu_baseline,
clocks, gpu_launches, the workload config (identical keys in both arms) and
the engine's own measurements under `detail`.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "CP-ALS sec/iter"
UNIT = "s/iter"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="engine", choices=["engine", "reference"])
    p.add_argument("--config", type=int, default=4)
    p.add_argument("--scale", type=float, default=1.0)
    p.add_argument("--rank", type=int, default=32)
    p.add_argument("--path", default="auto", choices=["auto", "tf32", "fp64"])
    p.add_argument("--threshold", type=float, default=0.03)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--keep-tns", default="", help="reference arm: keep the .tns it writes here")
    p.add_argument("--ref-log", default="", help="reference arm: save cpTC's stdout here")
    p.add_argument("--exchange", default="nccl", choices=["nccl"],
                   help="how the ranks combine a mode update (several GPUs): one NCCL "
                        "all-reduce per mode update")
    p.add_argument("--e2e-replicated", action="store_true",
                   help="e2e on several GPUs: every rank uploads and reads back whole factors "
                        "(default: each rank moves its 1/G of every factor and the pieces are "
                        "all-gathered on the GPUs, cptc_set_factors_sharded)")
    p.add_argument("--no-r128", action="store_true",
                   help="skip the R=128 sub-record of an R=32 run")
    p.add_argument("--phases", type=int, default=0,
                   help="after the timed steps, run this many iterations with per-phase "
                        "timing events and report their mean phase times per rank")
    return p.parse_args()


def workload_name(a) -> str:
    names = {1: "cfg1 128^3 200K uniform", 2: "cfg2 256^3 15.1M", 3: "cfg3 512^3 20M tiles+res",
             4: "cfg4 12092x9184x28818 76.9M Zipf(1.1) lognormal", 5: "cfg5 183x24x1140x1717 3.3M"}
    s = names.get(a.config, f"cfg{a.config}")
    if a.scale != 1.0:
        s += f" (nnz x{a.scale})"
    return f"{s}, CP-ALS R={a.rank}"


L2_NOTE = "views (1.2 GB/mode) stream from HBM each MTTKRP; no flush needed"


def shared_config(a, nnz: int, dims) -> dict:
    """The workload as both arms state it (same keys, same values): which
    tensor, rank and cutoff; measurements go elsewhere in the line."""
    return {"workload": workload_name(a), "rank": a.rank, "nnz": int(nnz),
            "dims": [int(d) for d in dims], "threshold": a.threshold, "seed": 0,
            "l2": L2_NOTE}


def want_r128(a) -> bool:
    return a.rank == 32 and not a.no_r128


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self._nv, self._h = nv, h
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((sm, rs))
            except Exception:
                pass
            time.sleep(0.005)

    def stop(self) -> dict:
        self._stop.set()
        if self._t:
            self._t.join()
        if not self._nv or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        nv = self._nv
        names = {
            "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
            "hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
            "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
            "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
            "hw_power_brake_slowdown": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown,
        }
        seen = set()
        for _, rs in self.samples:
            for k, bit in names.items():
                if rs & bit:
                    seen.add(k)
        return {"sm_mhz": float(np.median([s for s, _ in self.samples])),
                "sm_max_mhz": float(self.max_mhz), "reasons": sorted(seen),
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# tensor generation (rank 0 generates, other ranks read the shared copy)
# ---------------------------------------------------------------------------
def _cache_path(a) -> Path:
    d = Path(tempfile.gettempdir()) / "cptc_bench_cache"
    d.mkdir(exist_ok=True)
    return d / f"cfg{a.config}_s{a.scale}.npz"


def load_or_generate(a):
    """The seeded workload; cached as .npz in the temp folder because
    generating the 76.9M-nonzero tensor takes tens of seconds."""
    import cptc_b200 as cp

    path = _cache_path(a)
    if path.exists():
        z = np.load(path)
        dims = tuple(int(x) for x in z["dims"])
        return cp.CooTensor(dims, [z[f"i{m}"] for m in range(len(dims))], z["vals"])
    t = cp.gen_config(a.config, a.scale)
    tmp = path.with_suffix(".tmp.npz")
    np.savez(tmp, dims=np.array(t.dims, dtype=np.uint64), vals=t.vals,
             **{f"i{m}": t.idx[m] for m in range(t.order)})
    os.replace(tmp, path)
    return t


def get_tensor(a, rank: int, world: int, barrier):
    if world == 1:
        return load_or_generate(a)
    if rank == 0:
        t = load_or_generate(a)
        barrier()
        return t
    barrier()
    return load_or_generate(a)


def algorithmic_bytes(nnz: int, order: int, R: int, rows: int) -> int:
    """Bytes of one FP64 sparse MTTKRP per the survey's accounting: value,
    N-1 indices and N-1 gathered factor rows per nonzero, output written
    once."""
    return nnz * (8 + 4 * (order - 1) + 8 * R * (order - 1)) + 8 * R * rows


TF32_NOMINAL_TFLOPS = 1100.0  # B200 dense TF32, nominal


def tile_tflops(st, R: int, tile_ms) -> float | None:
    """TF32 MMA rate of the dense-tile kernel: 8192*R flops per tile per mode."""
    ms = float(np.mean(tile_ms)) if len(tile_ms) else 0.0
    if not st["tf32_path"] or ms <= 0.0:
        return None
    return st["dense_tiles"] * 8192.0 * R / (ms / 1000.0) / 1e12


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def cpu_baseline(t, R: int) -> dict:
    """The oracle (C++ COO MTTKRP, all host threads) on the same tensor: the
    three MTTKRPs of one ALS iteration, which are >95% of its CPU time."""
    from oracle import oracle as o

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    F = [rng.random((d, R)) for d in t.dims]
    t0 = time.perf_counter()
    for n in range(t.order):
        o.mttkrp(t, F, n, threads=threads)
    dt = time.perf_counter() - t0
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            model = next((ln.split(":", 1)[1].strip() for ln in f
                          if ln.startswith("model name")), "")
    except OSError:
        pass
    return {"value": dt, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": model,
            "sample": f"one ALS iteration's {t.order} FP64 MTTKRPs on the full tensor "
                      f"(oracle/cptc_oracle.cpp, OpenMP {threads} threads)"}


# ---------------------------------------------------------------------------
# engine arm
# ---------------------------------------------------------------------------
def pinned(shape):
    """float64 host array in page-locked memory (torch's pinned allocator)."""
    import torch

    return torch.empty(shape, dtype=torch.float64, pin_memory=True).numpy()


def run_engine(a):
    import cptc_b200 as cp
    from cptc_b200.engine import launch_count

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if dist is not None:
            dist.barrier()

    t = get_tensor(a, rank, world, barrier)
    eng = cp.Engine(local)
    if world > 1:
        uid = cp.comm_unique_id() if rank == 0 else None
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        eng.comm_init(obj[0], rank, world)

    # ---- end to end through the C ABI: host COO in, factors out ----------
    tb0 = time.perf_counter()
    eng.load(t)
    tb1 = time.perf_counter()
    eng.build(a.rank, threshold=a.threshold, path=a.path, exchange=a.exchange)
    eng.init_factors()
    build_s = time.perf_counter() - tb0
    load_s = tb1 - tb0
    st = eng.stats()

    # warm-up iterations (also the e2e steps' starting point); the first one
    # (graph capture included) is reported apart
    warm = eng.als(a.warmup)
    first_iter_ms = warm[0].ms if warm else None

    # ---- device-timed steps (inputs resident) ------------------------------
    barrier()
    clk = ClockSampler(local).start()
    l0 = launch_count()
    reps = eng.als(a.steps)
    l1 = launch_count()
    clocks = clk.stop()
    dev_s = sum(r.ms for r in reps) / 1000.0
    mode_ms = np.mean([r.mode_ms for r in reps], axis=0).tolist()
    fits = [r.fit for r in reps]

    # ---- e2e steps: factors from pinned host memory, ALS step, factors and
    # fit back to host, all through the C ABI ---------------------------------
    # Host buffers are pinned, as an application streaming factors would keep them.
    host_F = [pinned((t.dims[m], a.rank)) for m in range(t.order)]
    host_lam = pinned((a.rank,))
    for m in range(t.order):
        eng.factor(m, out=host_F[m])
    h2d = sum(f.nbytes for f in host_F)
    barrier()
    te0 = time.perf_counter()
    sharded = (not a.e2e_replicated) and world > 1
    for _ in range(a.steps):
        for m in range(t.order):
            eng.set_factor(m, host_F[m], sharded=sharded)
        eng.als(1)
        # every rank reads the step's result back (its replica; sharded: its
        # 1/G of the rows, the ones it uploads next), so every rank starts
        # the next step from the same factors
        for m in range(t.order):
            eng.factor(m, out=host_F[m], sharded=sharded)
        eng.lam(out=host_lam)
    e2e_s = (time.perf_counter() - te0) / a.steps
    fbytes = sum(f.nbytes for f in host_F)
    if not sharded:
        h2d *= world  # every rank uploads its replica
    d2h = (fbytes if sharded else fbytes * world) + (host_lam.nbytes + 16) * world

    # ---- per-phase times of each mode update (diagnostic, untimed) ---------
    phase_ms = None
    if a.phases > 0:
        eng.set_phase_timing(True)
        eng.als(1)  # the iteration graph is captured again with the events
        ph = [r.phases for r in eng.als(a.phases)]
        eng.set_phase_timing(False)
        phase_ms = np.mean(ph, axis=0)

    # ---- roofline of the dominant kernel -----------------------------------
    prof = [eng.profile_mttkrp(n, reps=3) for n in range(t.order)]
    rank_mode_ms = None
    shards = None
    rank_phase_ms = None
    rank_kernel_ms = None
    kern_ms = np.array([[p["sparse_ms"], p["tiles_ms"]] for p in prof])  # (modes, 2)
    gceil = gather_ceiling(eng, local, t, st["sparse_nnz"], a.rank, [p["sparse_ms"] for p in prof])
    if phase_ms is not None:
        rank_phase_ms = [np.round(phase_ms, 4).tolist()]
        rank_kernel_ms = [np.round(kern_ms, 4).tolist()]

    # ---- R=128 sub-record: the metric's second rank, same tensor ----------
    r128 = None
    if want_r128(a):
        eng.build(128, threshold=a.threshold, path=a.path, exchange=a.exchange)
        eng.init_factors()
        eng.als(a.warmup)
        barrier()
        # as many iterations as the reference arm runs, so that the final
        # fits of the two arms are taken after the same iteration
        reps128 = eng.als(a.steps)
        prof128 = [eng.profile_mttkrp(n, reps=2) for n in range(t.order)]
        st128 = eng.stats()
        r128 = {"ms_per_iter": float(np.mean([r.ms for r in reps128])),
                "iters": len(reps128),
                "mttkrp_ms_per_mode": np.mean([r.mode_ms for r in reps128], axis=0).tolist(),
                "sparse_kernel_ms_per_mode": [p["sparse_ms"] for p in prof128],
                "tile_kernel_ms_per_mode": [p["tiles_ms"] for p in prof128],
                "final_fit": reps128[-1].fit,
                "fit_iters": a.warmup + len(reps128),
                "tf32_path": bool(st128["tf32_path"])}
        r128["gather_ceiling"] = gather_ceiling(eng, local, t, st128["sparse_nnz"], 128,
                                                r128["sparse_kernel_ms_per_mode"])

    if dist is not None:
        import torch

        v = torch.tensor([dev_s, e2e_s, r128["ms_per_iter"] if r128 else 0.0],
                         dtype=torch.float64)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        dev_s, e2e_s = float(v[0]), float(v[1])
        if r128:
            r128["ms_per_iter"] = float(v[2])  # max over ranks
        # per-rank MTTKRP times (the iteration waits for the slowest rank)
        mm = torch.tensor(mode_ms, dtype=torch.float64)
        gathered = [torch.zeros_like(mm) for _ in range(world)]
        dist.all_gather(gathered, mm)
        rank_mode_ms = [[round(float(x), 4) for x in g] for g in gathered]
        if phase_ms is not None:
            pm = torch.tensor(phase_ms, dtype=torch.float64)
            pg = [torch.zeros_like(pm) for _ in range(world)]
            dist.all_gather(pg, pm)
            rank_phase_ms = [np.round(g.numpy(), 4).tolist() for g in pg]
            # this rank's share of the residual and tile kernels, per mode
            km = torch.tensor(kern_ms, dtype=torch.float64)
            kg = [torch.zeros_like(km) for _ in range(world)]
            dist.all_gather(kg, km)
            rank_kernel_ms = [np.round(g.numpy(), 4).tolist() for g in kg]
        # each rank's share of every mode's MTTKRP (residual nonzeros, rows,
        # tiles, tile words)
        mine = {k: list(st[k]) for k in ("local_sparse_nnz", "local_rows", "local_tiles",
                                         "local_tile_words")}
        shards = [None] * world
        dist.all_gather_object(shards, mine)

    if rank != 0:
        eng.close()
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    value = dev_s / a.steps
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": value * 1000.0,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f64+tf32" if st["tf32_path"] else "f64",
        "data": "synthetic (seeded generator, cptc_gen_config)",
        "config": shared_config(a, t.nnz, t.dims),
        "detail": {
            "path": "tf32 dense tiles + fp64 residual" if st["tf32_path"] else "fp64",
            "dense_tiles": st["dense_tiles"],
            "dense_nnz": st["dense_nnz"],
            "sparse_nnz": st["sparse_nnz"],
            "avg_fill": st["avg_fill"],
            "parallelism": f"row-slab x{world}" if world > 1 else "single GPU",
            "exchange": a.exchange if world > 1 else None,
            "build_s": build_s,
            "load_s": load_s,
            "device_build_ms": st["build_ms"],
            "first_iter_ms": first_iter_ms,
            "mttkrp_ms_per_mode": mode_ms,
            "mttkrp_ms_per_mode_by_rank": rank_mode_ms if world > 1 else None,
            "phase_ms_by_rank": rank_phase_ms,
            "phase_names": list(cp.Engine.PHASES) if rank_phase_ms is not None else None,
            "residual_tile_ms_by_rank": rank_kernel_ms,
            "shard_by_rank": shards,
            "final_fit": fits[-1],
        },
        "r128": r128,
        "e2e": {"value": e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "upload": ("each rank 1/G, all-gathered on the GPUs" if sharded else
                           "every rank its whole replica" if world > 1 else "whole factors")},
        "gpu_launches": int(l1 - l0),
        "clocks": clocks,
        "roofline": roofline_record(a, t, st, prof),
    }
    line["roofline"]["gather_ceiling"] = gceil
    if not a.no_cpu_baseline and world == 1:  # measured at N=1 only
        line["cpu_baseline"] = cpu_baseline(t, a.rank)
    print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def recorded_traffic(a):
    """ncu DRAM bytes per launch of the dominant kernel for this workload
    (profiles/traffic.json), or None."""
    prof_file = ROOT / "profiles" / "traffic.json"
    if not prof_file.exists() or a.scale != 1.0:
        return None  # recorded for the full-size workload only
    try:
        return json.loads(prof_file.read_text()).get(f"cfg{a.config}_R{a.rank}")
    except Exception:
        return None


def gather_ceiling(eng, device, t, nnz_view, R, sparse_ms) -> dict:
    """The residual kernel against the floor set by its own memory accesses.

    `replay_ms_per_mode`: a gather-only replay of each mode's residual
    MTTKRP (the same tasks, records and factor rows with the same lane layout,
    no arithmetic; cptc_profile_gather), beside the kernel's own time;
    `frac` = replay time / kernel time.  `uniform_probe_gbs`: uniformly random
    R-wide rows of an L2-resident matrix of the longest mode's size
    (cptc_gather_peak), the rate such gathers reach without the tensor's
    locality; `kernel_row_gbs` counts one row per nonzero at the kernel's
    rate (the outer rows, reused along fibers, are mostly L1 hits)."""
    import cptc_b200 as cp

    out = {"unit": "ms"}
    if t.order == 3:
        g = [eng.profile_gather(n, reps=3) for n in range(t.order)]
        rep = [x["replay_ms"] for x in g]
        ker = [x["kernel_ms"] for x in g]
        out.update({"replay_ms_per_mode": rep, "kernel_ms_per_mode": ker,
                    "frac": float(np.sum(rep) / np.sum(ker)) if np.sum(ker) > 0 else None})
    rows = int(max(t.dims))
    peak = cp.gather_peak(device, rows, R, max(int(nnz_view), 1 << 20), reps=3)
    ktime = float(np.mean(sparse_ms)) / 1000.0
    out.update({"uniform_probe_gbs": peak,
                "kernel_row_gbs": nnz_view * 8.0 * R / ktime / 1e9 if ktime > 0 else None,
                "uniform_probe": f"uniformly random rows of an L2-resident {rows}x{R} FP64 "
                                 "matrix, the kernel's row layout (cptc_gather_peak)"})
    return out


def roofline_record(a, t, st, prof) -> dict:
    """Roofline of the dominant kernel (the FP64 residual MTTKRP).

    `achieved` counts the bytes the kernel must move from HBM at least (its
    record stream once, each factor matrix it reads once, each output row
    once) per launch, over the kernel's mean CUDA-event duration; `frac` is
    that rate over the measured HBM copy bandwidth.  The bytes the kernel's
    factor-row gathers move through L1/L2 (a row per use) are reported apart,
    as `gather_bytes_per_launch` and `gather_rate_gbs`."""
    sp = [p["sparse_ms"] for p in prof]
    tl = [p["tiles_ms"] for p in prof]
    dominant = "k_mttkrp_rec3s" if t.order == 3 else "k_mttkrp_view"
    nnz_view = st["sparse_nnz"]
    rec_bytes = 16 if t.order == 3 else 32
    comp = [rec_bytes * nnz_view + 8 * a.rank * (sum(t.dims) - t.dims[n]) + 8 * a.rank * t.dims[n]
            for n in range(t.order)]
    gath = [algorithmic_bytes(nnz_view, t.order, a.rank, t.dims[n]) for n in range(t.order)]
    comp_launch = float(np.mean(comp))
    gath_launch = float(np.mean(gath))
    ktime = float(np.mean(sp)) / 1000.0
    peaks = measured_peaks()
    achieved = comp_launch / ktime / 1e9 if ktime > 0 else None
    tf = tile_tflops(st, a.rank, tl)
    return {
        "bound": "hbm",
        "kernel": dominant,
        "achieved": achieved,
        "peak": peaks["hbm_gbs"],
        "unit": "GB/s",
        "frac": (achieved / peaks["hbm_gbs"]) if achieved else None,
        "peak_src": peaks["src"],
        "traffic": recorded_traffic(a),
        "algorithmic_bytes_per_launch": comp_launch,
        "bytes_note": "algorithmic = compulsory HBM bytes per launch (record stream once, "
                      "factor matrices once, output rows once); the survey's gather-counted "
                      "bytes are gather_bytes_per_launch, moved through L1/L2",
        "gather_bytes_per_launch": gath_launch,
        "gather_rate_gbs": gath_launch / ktime / 1e9 if ktime > 0 else None,
        "sparse_kernel_ms_per_mode": sp,
        "tile_kernel_ms_per_mode": tl,
        "tile_tflops": tf,
        # no measured TF32 peak exists for this pool: nominal dense TF32
        "tile_tf32_frac_of_nominal": (tf / TF32_NOMINAL_TFLOPS) if tf else None,
    }


# ---------------------------------------------------------------------------
# reference arm: cpTC's own sources rebuilt for sm_100a (oracle/_ref)
# ---------------------------------------------------------------------------
def parse_ref_log(out: str):
    times, fits = [], []
    for ln in out.splitlines():
        if ln.startswith("[ALS] iter ") or ln.startswith("[GEN] iter "):
            parts = dict(kv.split("=") for kv in ln.split() if "=" in kv)
            times.append(float(parts["time"]))
            fits.append(float(parts["fit"]))
    return times, fits


def run_ref_binary(a, binary: Path, tns: Path, R: int, order: int):
    """cpTC on `tns` for warmup + steps iterations; (timed ms list, fits,
    selector line, stdout) or raises RuntimeError with its exit status."""
    env = dict(os.environ)
    if order != 3:
        # config 5's switches: HITS relabelling (3 rounds), dense units at
        # the cutoff of the run
        env.update({"GEN_REORDER": "hits", "GEN_REORDER_T": "3",
                    "GEN_DENSE_THRESHOLD": str(a.threshold)})
    iters = a.warmup + a.steps
    r = subprocess.run([str(binary), str(tns), str(iters), str(R), str(a.threshold)],
                       capture_output=True, text=True, env=env, timeout=1800)
    if a.ref_log:
        with open(a.ref_log, "a") as f:
            f.write(f"=== R={R}\n" + r.stdout + "\n--- stderr ---\n" + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"cpTC exited {r.returncode}: {r.stderr.strip()[-200:]}")
    times, fits = parse_ref_log(r.stdout)
    selector = next((ln for ln in r.stdout.splitlines() if "avg_fill=" in ln), "")
    return times[a.warmup:], fits, selector


def run_reference_port(a):
    """Without cpTC's own build: the oracle's restatement of its order-3
    CP-ALS on all host cores, one iteration (CADR and init included) of the
    same tensor."""
    import cptc_b200 as cp
    from oracle import oracle as o

    t = cp.gen_config(a.config, a.scale)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    o.cp_als3(t, a.rank, 1, thr=a.threshold, path="fp64", threads=threads)
    v = time.perf_counter() - t0
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
                      "higher_is_better": False, "n_gpus": 0, "steps": 1, "warmup": 0,
                      "config": shared_config(a, t.nnz, t.dims),
                      "cpu_baseline": {"kind": "port", "cores": threads, "value": v,
                                       "unit": UNIT,
                                       "sample": "one full CP-ALS iteration incl. CADR and init"},
                      "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


def run_reference(a):
    """The reference arm runs programs only: this repository's standalone
    generator (cptc_gen) writes the seeded tensor as .tns, then cpTC's own
    driver, rebuilt from its unmodified sources, reads and decomposes it.
    No library of this repository is loaded into this process."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    binary = ROOT / "oracle" / "_ref" / "cptc_opt"
    gen = ROOT / "cptc_b200" / "_lib" / "cptc_gen"
    if not binary.exists() or not gen.exists():
        run_reference_port(a)
        return
    with tempfile.TemporaryDirectory() as d:
        tns = Path(a.keep_tns) if a.keep_tns else Path(d) / "bench.tns"
        g = subprocess.run([str(gen), str(a.config), repr(a.scale), str(tns)],
                           capture_output=True, text=True, timeout=1800)
        if g.returncode != 0:
            print(json.dumps({"impl": "reference",
                              "unavailable": f"cptc_gen exited {g.returncode}: "
                                             f"{g.stderr.strip()[-200:]}"}))
            return
        info = json.loads(g.stdout.strip().splitlines()[-1])
        order, nnz, dims = info["order"], info["nnz"], info["nominal_dims"]
        try:
            timed, fits, selector = run_ref_binary(a, binary, tns, a.rank, order)
            r128 = None
            if want_r128(a):
                t128, f128, _ = run_ref_binary(a, binary, tns, 128, order)
                r128 = {"ms_per_iter": float(np.mean(t128)) if t128 else None,
                        "median_ms_per_iter": float(np.median(t128)) if t128 else None,
                        "iters": len(t128), "final_fit": f128[-1] if f128 else None,
                        "fit_iters": len(f128)}
        except RuntimeError as e:
            print(json.dumps({"impl": "reference", "unavailable": str(e)}))
            return
    v = float(np.mean(timed)) / 1000.0
    med = float(np.median(timed)) / 1000.0 if timed else None
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
            "higher_is_better": False, "n_gpus": 1, "steps": len(timed), "warmup": a.warmup,
            "ms_per_step": v * 1000.0, "median": med, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64+tf32",
            "data": "synthetic (same generator and seed, written as .tns by cptc_gen)",
            "config": shared_config(a, nnz, dims),
            "detail": {"selector_line": selector[:300], "final_fit": fits[-1] if fits else None,
                       "median_ms_per_step": med * 1000.0 if med else None,
                       "max_ms_per_step": max(timed) if timed else None,
                       "dims_read": info["dims"]},
            "r128": r128,
            "cpu_baseline": {"kind": "reference", "cores": 1, "value": v, "unit": UNIT,
                             "sample": "zhixianzhu/cpTC sources rebuilt for sm_100a "
                                       "(oracle/build_ref.sh), one host thread driving one "
                                       "B200; mean of the per-iteration times it prints "
                                       "([ALS] iter ... time=) after the warm-up iterations"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    a = parse_args()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_engine(a)


if __name__ == "__main__":
    main()
