"""bench.py's accounting on CPU: the algorithmic bytes of the sparse MTTKRP
(per nonzero: value, N-1 indices, N-1 gathered factor rows; each output row
once), the TF32 tile rate, the peak it divides by, and the CPU baseline's
report."""
import subprocess
import sys
from pathlib import Path

import pytest

import cptc_b200 as cp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_algorithmic_bytes_per_nonzero():
    # 8 + 8 + 16R bytes per nonzero at order 3, 8 + 12 + 24R at order 4
    assert bench.algorithmic_bytes(1, 3, 32, 0) == 528
    assert bench.algorithmic_bytes(1, 3, 128, 0) == 2064
    assert bench.algorithmic_bytes(1, 4, 16, 0) == 404
    # output rows once: 8R bytes each
    assert bench.algorithmic_bytes(0, 3, 32, 1000) == 8 * 32 * 1000
    # config 4 at R=32, whole iteration: ~121.8 GB over the three modes when
    # every nonzero is in the residual
    dims = (12092, 9184, 28818)
    per_iter = sum(bench.algorithmic_bytes(76_900_000, 3, 32, d) for d in dims)
    assert abs(per_iter / 1e9 - 121.8) < 0.2


def test_tile_rate():
    st = {"tf32_path": 1, "dense_tiles": 1000}
    # 1000 tiles x 8192 x 32 flops in 1 ms = 0.262 TFLOP/s
    assert abs(bench.tile_tflops(st, 32, [1.0, 1.0]) - 0.262144) < 1e-9
    assert bench.tile_tflops({"tf32_path": 0, "dense_tiles": 0}, 32, [1.0]) is None


def test_peak_source():
    p = bench.measured_peaks()
    assert p["hbm_gbs"] > 1000 and p["src"] in ("measured", "fallback")


def test_cpu_baseline_report():
    t = cp.gen_config(1, scale=0.05)
    r = bench.cpu_baseline(t, 8)
    assert r["kind"] == "port" and r["cores"] >= 1 and r["value"] > 0
    assert set(r) >= {"value", "unit", "cores", "kind", "sample"}


def test_cli_flags():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"],
                         capture_output=True, text=True, check=True).stdout
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--rank", "--exchange",
                 "--e2e-replicated", "--phases"):
        assert flag in out


@pytest.mark.parametrize("argv", [["--gpus", "2", "--steps", "3"], []])
def test_defaults_parse(argv, monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    a = bench.parse_args()
    assert a.warmup >= 3 and a.config == 4 and a.rank == 32 and a.exchange == "nccl"
