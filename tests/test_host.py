"""Host-side library: generators, .tns reader/writer, the C ABI exports."""
import ctypes as C
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import cptc_b200 as cp
from cptc_b200 import _native as N

ROOT = Path(__file__).resolve().parent.parent


def test_generator_deterministic_across_threads():
    env = dict(os.environ, CPTC_HOST_THREADS="1")
    code = ("import cptc_b200 as cp, hashlib; t = cp.gen_config(1); "
            "h = hashlib.sha1(); [h.update(a.tobytes()) for a in t.idx]; h.update(t.vals.tobytes()); "
            "print(h.hexdigest())")
    one = subprocess.run([sys.executable, "-c", code], env=env, cwd=ROOT, capture_output=True,
                         text=True, check=True).stdout.strip()
    env["CPTC_HOST_THREADS"] = "5"
    five = subprocess.run([sys.executable, "-c", code], env=env, cwd=ROOT, capture_output=True,
                          text=True, check=True).stdout.strip()
    assert one == five


@pytest.mark.parametrize("cfg,scale", [(1, 1.0), (2, 0.01), (3, 0.005), (4, 0.001), (5, 0.01)])
def test_configs_distinct_and_in_range(cfg, scale):
    t = cp.gen_config(cfg, scale=scale)
    assert t.nnz > 0
    key = np.zeros(t.nnz, dtype=np.uint64)
    for m, d in enumerate(t.dims):
        assert t.idx[m].max() < d
        key = key * np.uint64(d) + t.idx[m].astype(np.uint64)
    assert len(np.unique(key)) == t.nnz  # distinct coordinates
    assert np.all(np.diff(key.astype(np.float64)) > 0)  # sorted by linear key


def test_config_shapes():
    assert cp.gen_config(4, scale=1e-4).dims == (12092, 9184, 28818)
    assert cp.gen_config(5, scale=1e-3).dims == (183, 24, 1140, 1717)
    t = cp.gen_config(1)
    assert t.nnz == 200000 and t.dims == (128, 128, 128)


def test_tns_roundtrip(tmp_path):
    t = cp.gen_uniform((30, 40, 7, 5), 3000, seed=9, values="lognormal")
    p = tmp_path / "x.tns"
    cp.write_tns(p, t)
    assert cp.probe_order(p) == 4
    u = cp.read_tns(p)
    assert u.dims == tuple(int(i.max()) + 1 for i in t.idx)
    for a, b in zip(t.idx, u.idx):
        assert np.array_equal(a, b)
    assert np.array_equal(t.vals, u.vals)  # %.17g is exact


def test_tns_parse_rules(tmp_path):
    p = tmp_path / "y.tns"
    p.write_text("# comment\n1 2 3 1.5\n\n  4\t5 6 -2e3\n0 1 1 7\n2 2 bad\n3 3 3\n9 1 1 x\n")
    t = cp.read_tns(p)
    assert t.order == 3
    assert t.nnz == 3  # lines without a parseable value are skipped
    assert t.idx[0].tolist() == [0, 3, 0]  # 1-based, index 0 maps to 0
    assert t.vals.tolist() == [1.5, -2000.0, 7.0]
    assert t.dims == (4, 5, 6)


def _declared(header: Path):
    txt = header.read_text()
    return set(re.findall(r"^\w[\w\s\*]*?\b(cptc_\w+)\s*\(", txt, flags=re.M))


def test_engine_library_exports_every_declared_symbol():
    lib_path = N.LIB_DIR / "libcptc.so"
    assert lib_path.exists(), "build the engine first (python -m cptc_b200.build)"
    lib = C.CDLL(str(lib_path))
    names = _declared(ROOT / "include" / "cptc.h") | _declared(ROOT / "include" / "cptc_host.h")
    assert "cptc_mttkrp" in names and "cptc_gen_config" in names
    for n in sorted(names):
        assert hasattr(lib, n), n
    # the Python binding table covers the same set
    assert names == set(N.HOST_SYMBOLS) | set(N.ENGINE_SYMBOLS)


def test_engine_loads_without_gpu_and_fails_loudly():
    lib = N.engine_lib()
    h = C.c_void_p()
    rc = lib.cptc_create(C.byref(h), 0, 0)
    try:
        import torch
        has = torch.cuda.is_available()
    except Exception:
        has = False
    if not has:
        assert rc != 0  # no silent CPU fallback
    else:
        assert rc == 0
        lib.cptc_destroy(h)


def test_bin_cache_roundtrip_and_reuse(tmp_path):
    t = cp.gen_uniform((30, 40, 7, 5), 3000, seed=9, values="lognormal")
    p = tmp_path / "x.tns"
    cp.write_tns(p, t)
    u, hit = cp.read_tns_cached(p)
    assert not hit and (tmp_path / "x.tns.cptcbin").exists()
    v, hit = cp.read_tns_cached(p)
    assert hit
    ref = cp.read_tns(p)
    for w in (u, v):
        assert w.dims == ref.dims
        for a, b in zip(w.idx, ref.idx):
            assert np.array_equal(a, b)
        assert np.array_equal(w.vals, ref.vals)
    # the probed order as a hint uses the cache; another hint parses the
    # text with that order (and caches that), after which the probed order
    # parses again
    assert cp.read_tns_cached(p, order=4)[1]
    w, hit = cp.read_tns_cached(p, order=3)
    assert not hit and w.order == 3
    assert cp.read_tns_cached(p, order=3)[1]
    w, hit = cp.read_tns_cached(p)
    assert not hit and w.order == 4


def test_bin_cache_is_stale_when_the_text_changes(tmp_path):
    p = tmp_path / "y.tns"
    p.write_text("1 2 3 1.5\n4 5 6 2.5\n")
    t, hit = cp.read_tns_cached(p)
    assert not hit and t.nnz == 2
    st = p.stat()
    p.write_text("1 2 3 1.5\n4 5 6 2.5\n7 1 1 3.0\n")
    os.utime(p, ns=(st.st_atime_ns, st.st_mtime_ns + 10**9))
    t, hit = cp.read_tns_cached(p)
    assert not hit and t.nnz == 3 and t.dims == (7, 5, 6)
    t, hit = cp.read_tns_cached(p)
    assert hit and t.nnz == 3


def test_bin_cache_rejects_corrupt_and_truncated_files(tmp_path):
    t = cp.gen_uniform((50, 60, 70), 5000, seed=3)
    b = tmp_path / "t.bin"
    cp.write_bin(b, t, 123, 456)
    u = cp.read_bin(b)
    assert u.dims == t.dims and np.array_equal(u.vals, t.vals)
    raw = bytearray(b.read_bytes())
    bad = tmp_path / "bad.bin"
    raw2 = bytearray(raw)
    raw2[len(raw2) - 5] ^= 0x40  # a value byte
    bad.write_bytes(bytes(raw2))
    with pytest.raises(RuntimeError, match="hash"):
        cp.read_bin(bad)
    bad.write_bytes(bytes(raw[:-8]))
    with pytest.raises(RuntimeError, match="truncated"):
        cp.read_bin(bad)
    bad.write_bytes(b"not a cache" * 20)
    with pytest.raises(RuntimeError):
        cp.read_bin(bad)
    # a corrupt sidecar is replaced by a parse of the text
    p = tmp_path / "z.tns"
    cp.write_tns(p, t)
    cp.read_tns_cached(p)
    side = tmp_path / "z.tns.cptcbin"
    raw = bytearray(side.read_bytes())
    raw[200] ^= 1
    side.write_bytes(bytes(raw))
    os.utime(side, ns=(p.stat().st_atime_ns, p.stat().st_mtime_ns))
    u, hit = cp.read_tns_cached(p)
    assert not hit and np.array_equal(u.vals, cp.read_tns(p).vals)
    assert cp.read_tns_cached(p)[1]


def test_bin_cache_hash_independent_of_threads(tmp_path):
    code = ("import cptc_b200 as cp, sys; t = cp.gen_config(4, scale=0.02); "
            "cp.write_bin(sys.argv[1], t)")
    outs = []
    for th in ("1", "3"):
        f = tmp_path / f"c{th}.bin"
        env = dict(os.environ, CPTC_HOST_THREADS=th)
        subprocess.run([sys.executable, "-c", code, str(f)], env=env, cwd=ROOT, check=True)
        outs.append(f.read_bytes())
    assert outs[0] == outs[1]


def test_ctypes_structs_match_the_c_headers(tmp_path):
    # the Python mirrors of cptc_opts, cptc_stats and cptc_coo must have the
    # C layout (a field added on one side only shifts every later field)
    src = tmp_path / "sz.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "cptc.h"\n'
                   'int main(void) { printf("%zu %zu %zu %zu\\n", sizeof(cptc_opts), '
                   'sizeof(cptc_stats), sizeof(cptc_coo), offsetof(cptc_opts, exchange)); '
                   'return 0; }\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got == [C.sizeof(N.Opts), C.sizeof(N.Stats), C.sizeof(N.Coo), N.Opts.exchange.offset]
