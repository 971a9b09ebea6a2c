"""Test configuration: the `gpu` marker, repo imports and the builds both suites need."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def hk():
    """The product library, built in-tree if needed (nvcc cross-compiles without a GPU)."""
    from hyperkernel_b200 import build

    if not (ROOT / "hyperkernel_b200" / "libhk.so").exists():
        build.build()
    from hyperkernel_b200 import _lib

    _lib.lib()
    return _lib


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def cuda(hk):
    """The GPU tests run on a B200; without one they fail rather than skip."""
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    sm, major, minor = hk.device_info()
    assert major == 10, f"sm_{major}{minor}: these kernels are built for sm_100a"
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)


def pytest_sessionfinish(session, exitstatus):
    """With HK_ERR_REPORT set, writes the normwise and element-wise max-abs-rel figures of
    every floating-point comparison the GPU kernel tests made (JSON lines)."""
    path = os.environ.get("HK_ERR_REPORT")
    mod = sys.modules.get("test_kernels_gpu") or sys.modules.get("tests.test_kernels_gpu")
    if not path or mod is None:
        return
    import json

    with open(path, "w") as f:
        for test, norm, elem in getattr(mod, "ERRS", []):
            f.write(json.dumps({"test": test, "normwise": norm, "elementwise": elem}) + "\n")
