"""Regenerates tests/golden/rope_windows.json from the reference's RoPE fixture.

The reference pins its RoPE table builder (src/gpu/load.rs:824-846) with
tests/fixtures/rope.json (test at src/gpu/load.rs:1036-1053): for two tables it stores
four windows of raw little-endian f32 bytes (8 rows of 64 values each).  This script
copies those windows into a compact fixture so the tests need no access to the reference
checkout at run time:

    python tests/golden/make_rope_golden.py /path/to/reference/tests/fixtures/rope.json
"""
import json
import sys
from pathlib import Path

if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_rope_golden.py <reference checkout>/tests/fixtures/rope.json")
src = Path(sys.argv[1])
data = json.loads(src.read_text())
out = {"source": "reference tests/fixtures/rope.json (src/gpu/load.rs:1036-1053)", "tables": []}
for t in data["tables"]:
    f = t["fill"]
    out["tables"].append({
        "name": t["name"],
        "params": {k: f[k] for k in ("rows", "dim", "base", "original_seq_len", "factor",
                                     "beta_fast", "beta_slow")},
        "windows": [{"row": w["row"], "hex": w["bytes"]} for w in t["windows"]],
    })
dst = Path(__file__).with_name("rope_windows.json")
dst.write_text(json.dumps(out, indent=1) + "\n")
print(f"wrote {dst}")
