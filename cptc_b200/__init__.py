"""cptc_b200 — CP-ALS for sparse tensors on NVIDIA B200 (sm_100a).

The MTTKRP hot path of zhixianzhu/cpTC rebuilt B200-first: hand-written
sm_100a CUDA behind a C ABI (include/cptc.h), with this package as the
Python face.  Native libraries are built in-tree by ``python -m
cptc_b200.build``.
"""
from .tensor import (CooTensor, gen_config, gen_uniform, probe_order, read_bin, read_tns,
                     read_tns_cached, write_bin, write_tns)
from .engine import CptcError, Engine, IterReport, comm_unique_id, gather_peak

__all__ = [
    "CooTensor",
    "CptcError",
    "Engine",
    "IterReport",
    "comm_unique_id",
    "gen_config",
    "gather_peak",
    "gen_uniform",
    "probe_order",
    "read_bin",
    "read_tns",
    "read_tns_cached",
    "write_bin",
    "write_tns",
]
