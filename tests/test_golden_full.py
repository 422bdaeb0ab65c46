"""Full-size parity: the reference's own per-iteration fits on the benchmark's
full configs 2 (15.1M nonzeros, every tile dense), 3 (20M nonzeros, every tile
above the cutoff), 4 (76.9M nonzeros, R=32 and R=128) and 5 (3.3M nonzeros,
order 4, HITS + dense units), recorded on a B200 by the reference arm of
bench.py (tests/golden/extract_ref_fits.py has the command).

The reference itself varies by ~2e-6 between runs at R=32 (atomics and TF32
rounding; both runs are kept), so fits are compared per iteration within
1e-5, the bound the TF32 goldens use.  Config 2 is computed entirely on the
TF32 path (4096 tiles at fill 0.9): the accumulation order inside a TF32 MMA
instruction (m16n8k8 here, the reference's WMMA m16n16k8) is the hardware's,
and on this well-fitted model (fit 0.68) the difference moves the first
iterations by up to 3e-5 (7e-6 at iteration 23); it is held to the task's
fit bound, 1e-4.
"""
import json
import os
from pathlib import Path

import numpy as np
import pytest

import cptc_b200 as cp

GOLD = Path(__file__).resolve().parent / "golden"
TOL = 1e-5
TOL_CASE = {"full_cfg2_R32": 1e-4}


def load(name):
    return json.loads((GOLD / f"{name}.json").read_text())


_cache = {}


def full_tensor(cfg):
    """Config `cfg` at full size, each mode sized as max index + 1 (the
    reference's rule, src/tensor.cu:247-254)."""
    if cfg not in _cache:
        t = cp.gen_config(cfg)
        _cache[cfg] = cp.CooTensor(tuple(int(i.max()) + 1 for i in t.idx), t.idx, t.vals)
    return _cache[cfg]


def within(fits, g):
    ref = np.array(g["fits"][:len(fits)])
    lo, hi = ref.copy(), ref.copy()
    if "fits_other_run" in g:
        other = np.array(g["fits_other_run"][:len(fits)])
        lo, hi = np.minimum(lo, other), np.maximum(hi, other)
    f = np.asarray(fits)
    return float(np.max(np.maximum(lo - f, f - hi).clip(min=0.0)))


def test_oracle_matches_reference_full_cfg5(oracle):
    g = load("full_cfg5_R16")
    t = full_tensor(5)
    fits, _, _ = oracle.cp_als_generic(t, g["R"], 6, dense_thr=g["threshold"], solver="chol",
                                       threads=os.cpu_count() or 1)
    assert within(fits, g) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["full_cfg2_R32", "full_cfg3_R32", "full_cfg4_R32",
                                  "full_cfg4_R128", "full_cfg5_R16"])
def test_engine_matches_reference_full_size(gpu, name):
    g = load(name)
    t = full_tensor(g["cfg"])
    e = cp.Engine(0)
    e.load(t)
    e.build(g["R"], threshold=g["threshold"])  # the reference's defaults for this order
    st = e.stats()
    # the reference's partition lines
    if g["cfg"] == 2:
        assert st["dense_tiles"] == 4096 and st["sparse_nnz"] == 0
    elif g["cfg"] == 3:
        assert st["dense_tiles"] == 32768 and st["sparse_nnz"] == 0
    elif g["cfg"] == 4:
        assert st["dense_tiles"] == 81886 and st["sparse_nnz"] == 37821322
    else:
        assert st["dense_nnz"] == 1828748
    e.init_factors()
    fits = [r.fit for r in e.als(g["iters"])]
    e.close()
    assert within(fits, g) < TOL_CASE.get(name, TOL)
