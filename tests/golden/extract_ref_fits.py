"""Turns the output of the reference program on a full-size benchmark tensor
into a golden fixture: its per-iteration fits and partition summary lines.

The output comes from the reference arm of bench.py, run on a B200 with the
reference rebuilt from its own sources (oracle/build_ref.sh):

  python bench.py --impl reference --config C --rank R --ref-log LOG
  python tests/golden/extract_ref_fits.py LOG --cfg C --rank R --out tests/golden/NAME.json

The tensor is the seeded synthetic config C at full size (cptc_gen_config),
written as .tns and read by the reference; one .tns line per nonzero.
"""
import argparse
import json
import re
from pathlib import Path


def parse(text: str) -> dict:
    fits, times = [], []
    for ln in text.splitlines():
        if ln.startswith("[ALS] iter ") or ln.startswith("[GEN] iter "):
            kv = dict(t.split("=", 1) for t in ln.split() if "=" in t)
            fits.append(float(kv["fit"]))
            times.append(float(kv["time"]))
    notes = [ln.strip() for ln in text.splitlines()
             if re.search(r"Dense Tiles|dense:|reorder=|avg_fill=", ln)]
    return {"fits": fits, "times_ms": times, "notes": notes}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("log")
    ap.add_argument("--cfg", type=int, required=True)
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--threshold", type=float, default=0.03)
    ap.add_argument("--out", required=True)
    ap.add_argument("--also", default="", help="a second run's log, kept as fits_other_run")
    a = ap.parse_args()
    rec = {"cfg": a.cfg, "scale": 1.0, "R": a.rank, "threshold": a.threshold}
    rec.update(parse(Path(a.log).read_text()))
    rec["iters"] = len(rec["fits"])
    if a.also:
        rec["fits_other_run"] = parse(Path(a.also).read_text())["fits"]
    rec["env"] = ({"GEN_REORDER": "hits", "GEN_REORDER_T": "3",
                   "GEN_DENSE_THRESHOLD": str(a.threshold)} if a.cfg == 5 else {})
    Path(a.out).write_text(json.dumps(rec, indent=1) + "\n")


if __name__ == "__main__":
    main()
