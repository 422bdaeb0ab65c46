"""Full-size parity: the reference's own per-iteration fits on the benchmark's
full config 4 (76.9M nonzeros, R=32 and R=128) and config 5 (3.3M nonzeros,
order 4, HITS + dense units), recorded on a B200 by the reference arm of
bench.py (tests/golden/extract_ref_fits.py has the command).

The reference itself varies by ~2e-6 between runs at R=32 (atomics and TF32
rounding; both runs are kept), so fits are compared per iteration within
1e-5, the bound the TF32 goldens use; the final-fit bound of the task is 1e-4.
"""
import json
import os
from pathlib import Path

import numpy as np
import pytest

import cptc_b200 as cp

GOLD = Path(__file__).resolve().parent / "golden"
TOL = 1e-5


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
@pytest.mark.parametrize("name", ["full_cfg4_R32", "full_cfg4_R128", "full_cfg5_R16"])
def test_engine_matches_reference_full_size(gpu, name):
    g = load(name)
    t = full_tensor(g["cfg"])
    e = cp.Engine(0)
    e.load(t)
    e.build(g["R"], threshold=g["threshold"])  # the reference's defaults for this order
    st = e.stats()
    if g["cfg"] == 4:
        # the reference's partition line: 81886 tiles, 37821322 residual nonzeros
        assert st["dense_tiles"] == 81886 and st["sparse_nnz"] == 37821322
    else:
        assert st["dense_nnz"] == 1828748
    e.init_factors()
    fits = [r.fit for r in e.als(g["iters"])]
    e.close()
    assert within(fits, g) < TOL
