"""CPU-side checks of the product library: it loads, exports every entry point of
include/hk.h, reports a missing device as an error (no CPU fallback), and its host-side
RoPE table matches the reference's fixture bytes."""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).parent / "golden" / "rope_windows.json"


def test_every_header_function_is_exported(hk):
    names = hk.header_functions()
    assert len(names) >= 20, names
    lib = C.CDLL(str(hk.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared in include/hk.h but not exported: {missing}"
    assert set(names) == set(hk.SIGNATURES), "ctypes prototypes out of step with include/hk.h"


def test_every_header_function_has_a_reference_side_binding(hk):
    """The integration guide at the repository root shows the Rust declaration a maintainer
    adds for each entry point."""
    text = (Path(__file__).resolve().parents[1] / "INTEGRATION.md").read_text()
    missing = [n for n in hk.header_functions() if f"fn {n}(" not in text]
    assert not missing, f"no Rust binding shown for: {missing}"


def test_version_and_no_device_is_an_error(hk):
    import torch

    assert "sm_100a" in hk.version()
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    sm, ma, mi = C.c_int(), C.c_int(), C.c_int()
    rc = hk.lib().hk_device_info(C.byref(sm), C.byref(ma), C.byref(mi))
    assert rc != 0 and hk.last_error()


def test_entry_points_refuse_without_a_device(hk):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc = hk.lib().hk_check_errors()
    assert rc in (hk.HK_ENODEV, hk.HK_ECUDA), rc


def _windows():
    data = json.loads(GOLDEN.read_text())
    for t in data["tables"]:
        yield t["name"], t["params"], t["windows"]


@pytest.mark.parametrize("name", ["rope.window", "rope.pooled"])
def test_rope_table_matches_reference_fixture(hk, name):
    for n, p, windows in _windows():
        if n != name:
            continue
        rows = max(w["row"] for w in windows) + 8
        table = hk.rope_table(rows, p["dim"], p["base"], p["original_seq_len"], p["factor"],
                              p["beta_fast"], p["beta_slow"])
        for w in windows:
            want = bytes.fromhex(w["hex"])
            got = table[w["row"]:].tobytes()[:len(want)]
            assert got == want, f"{name} row {w['row']}"
