#!/usr/bin/env python
"""CP-ALS benchmark: seconds per ALS iteration on BASELINE config 4.

Workload: order-3 synthetic tensor 12092 x 9184 x 28818 with 76.9M nonzeros,
Zipf(1.1) indices per mode over a random permutation, lognormal values
(cptc_gen_config(4)); CP rank R=32 (R=128 with --rank 128); one step = one
CP-ALS iteration (3 mode updates + Gram fit).  The tensor views are streamed
from HBM every MTTKRP (1.2 GB per mode, larger than the 126 MB L2), so no
explicit L2 flush is needed between steps.

  python bench.py [--gpus N --steps K --warmup W --rank R]
  python bench.py --impl reference ...   # cpTC's own build (oracle/_ref)

One JSON line on rank 0: metric, value, unit, e2e, roofline, cpu_baseline,
clocks, gpu_launches and the workload config.
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
    p.add_argument("--exchange", default="nccl", choices=["nccl", "peer"],
                   help="how the ranks combine a mode update (several GPUs)")
    p.add_argument("--e2e-sharded", action="store_true",
                   help="e2e on several GPUs: each rank uploads 1/G of every factor and the "
                        "pieces are all-gathered on the GPUs (cptc_set_factors_sharded)")
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
    sharded = a.e2e_sharded and world > 1
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
    rank_phase_ms = None
    rank_kernel_ms = None
    kern_ms = np.array([[p["sparse_ms"], p["tiles_ms"]] for p in prof])  # (modes, 2)
    if phase_ms is not None:
        rank_phase_ms = [np.round(phase_ms, 4).tolist()]
        rank_kernel_ms = [np.round(kern_ms, 4).tolist()]

    if dist is not None:
        import torch

        v = torch.tensor([dev_s, e2e_s], dtype=torch.float64)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        dev_s, e2e_s = float(v[0]), float(v[1])
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

    if rank != 0:
        eng.close()
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    sp = [p["sparse_ms"] for p in prof]
    tl = [p["tiles_ms"] for p in prof]
    dominant = "k_mttkrp_rec3s" if t.order == 3 else "k_mttkrp_view"
    nnz_view = st["sparse_nnz"]
    # Per launch (one mode): the benchmark's algorithmic bytes (every factor-row
    # gather) and the compulsory bytes (each stored byte once).
    algo = [algorithmic_bytes(nnz_view, t.order, a.rank, t.dims[n]) for n in range(t.order)]
    comp = 16 * nnz_view + 8 * a.rank * sum(t.dims)
    algo_launch = float(np.mean(algo))
    ktime = float(np.mean(sp)) / 1000.0
    peaks = measured_peaks()
    achieved = algo_launch / ktime / 1e9 if ktime > 0 else None
    traffic = None
    prof_file = ROOT / "profiles" / "traffic.json"
    if prof_file.exists():
        try:
            traffic = json.loads(prof_file.read_text()).get(f"cfg{a.config}_R{a.rank}")
        except Exception:
            traffic = None
        if traffic is not None and a.scale != 1.0:
            traffic = None  # recorded for the full-size workload only

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
        "config": {
            "workload": workload_name(a),
            "rank": a.rank,
            "nnz": t.nnz,
            "dims": list(t.dims),
            "path": "tf32 dense tiles + fp64 residual" if st["tf32_path"] else "fp64",
            "dense_tiles": st["dense_tiles"],
            "dense_nnz": st["dense_nnz"],
            "avg_fill": st["avg_fill"],
            "parallelism": f"row-slab x{world}" if world > 1 else "single GPU",
            "exchange": a.exchange if world > 1 else None,
            "l2": "views (1.2 GB/mode) stream from HBM each MTTKRP; no flush needed",
            "build_s": build_s,
            "load_s": load_s,
            "device_build_ms": st["build_ms"],
            "first_iter_ms": first_iter_ms,
            "mttkrp_ms_per_mode": mode_ms,
            "mttkrp_ms_per_mode_by_rank": rank_mode_ms if world > 1 else None,
            "phase_ms_by_rank": rank_phase_ms,
            "phase_names": list(cp.Engine.PHASES) if rank_phase_ms is not None else None,
            "residual_tile_ms_by_rank": rank_kernel_ms,
            "final_fit": fits[-1],
        },
        "e2e": {"value": e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "upload": ("each rank 1/G, all-gathered on the GPUs" if sharded else
                           "every rank its whole replica" if world > 1 else "whole factors")},
        "gpu_launches": int(l1 - l0),
        "clocks": clocks,
        "roofline": {
            "bound": "hbm",
            "kernel": dominant,
            "achieved": achieved,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": (achieved / peaks["hbm_gbs"]) if achieved else None,
            "peak_src": peaks["src"],
            "traffic": traffic,
            "algorithmic_bytes_per_launch": algo_launch,
            "bytes_note": "algorithmic bytes count every factor-row gather; "
                          "most gathers hit L1/L2, so frac can exceed 1; compulsory_frac "
                          "counts each stored byte once",
            "compulsory_bytes_per_launch": comp,
            "compulsory_frac": (comp / ktime / 1e9 / peaks["hbm_gbs"]) if ktime > 0 else None,
            "sparse_kernel_ms_per_mode": sp,
            "tile_kernel_ms_per_mode": tl,
            "tile_tflops": tile_tflops(st, a.rank, tl),
            # no measured TF32 peak exists for this pool: nominal dense TF32
            "tile_tf32_frac_of_nominal": (tile_tflops(st, a.rank, tl) / TF32_NOMINAL_TFLOPS
                                          if tile_tflops(st, a.rank, tl) else None),
        },
    }
    if not a.no_cpu_baseline and world == 1:  # measured at N=1 only
        line["cpu_baseline"] = cpu_baseline(t, a.rank)
    print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# reference arm: cpTC's own sources rebuilt for sm_100a (oracle/_ref)
# ---------------------------------------------------------------------------
def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import cptc_b200 as cp

    binary = ROOT / "oracle" / "_ref" / "cptc_opt"
    t = load_or_generate(a)
    if not binary.exists():
        # Oracle port on the host cores instead.
        from oracle import oracle as o

        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        fits, _, _ = o.cp_als3(t, a.rank, 1, thr=a.threshold, path="fp64", threads=threads)
        v = time.perf_counter() - t0
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
                "higher_is_better": False, "n_gpus": 0, "steps": 1, "warmup": 0,
                "config": {"workload": workload_name(a)},
                "cpu_baseline": {"kind": "port", "cores": threads, "value": v, "unit": UNIT,
                                 "sample": "one full CP-ALS iteration incl. CADR and init"},
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    with tempfile.TemporaryDirectory() as d:
        tns = Path(a.keep_tns) if a.keep_tns else Path(d) / "bench.tns"
        cp.write_tns(tns, t)
        iters = a.warmup + a.steps
        env = dict(os.environ)
        if t.order != 3:
            # config 5's switches: HITS relabelling (3 rounds), dense units
            # at cutoff 0.03
            env.update({"GEN_REORDER": "hits", "GEN_REORDER_T": "3",
                        "GEN_DENSE_THRESHOLD": str(a.threshold)})
        r = subprocess.run([str(binary), str(tns), str(iters), str(a.rank), str(a.threshold)],
                           capture_output=True, text=True, env=env, timeout=1800)
        out = r.stdout
    if a.ref_log:
        Path(a.ref_log).write_text(out + "\n--- stderr ---\n" + r.stderr)
    if r.returncode != 0:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"cpTC exited {r.returncode}: {r.stderr.strip()[-200:]}"}))
        return
    times, fits = [], []
    for ln in out.splitlines():
        if ln.startswith("[ALS] iter ") or ln.startswith("[GEN] iter "):
            parts = dict(kv.split("=") for kv in ln.split() if "=" in kv)
            times.append(float(parts["time"]))
            fits.append(float(parts["fit"]))
    timed = times[a.warmup:]
    v = float(np.mean(timed)) / 1000.0
    med = float(np.median(timed)) if timed else None
    selector = next((ln for ln in out.splitlines() if "avg_fill=" in ln), "")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
            "higher_is_better": False, "n_gpus": 1, "steps": len(timed), "warmup": a.warmup,
            "ms_per_step": v * 1000.0, "scaling": "strong", "vs_baseline": None,
            "dtype": "f64+tf32", "data": "synthetic (same generator and seed)",
            "config": {"workload": workload_name(a), "rank": a.rank, "nnz": t.nnz,
                       "selector_line": selector[:300], "final_fit": fits[-1] if fits else None,
                       "median_ms_per_step": med, "max_ms_per_step": max(timed) if timed else None},
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
