"""Shared test setup: package path, the `gpu` marker, device helpers.

`-m "not gpu"` tests need no GPU (oracle vs golden vectors, host logic, C-ABI
symbol exports). `-m gpu` tests call the sm_100a kernels through the C-ABI
and compare them with the CPU oracle (oracle/).
"""

import ctypes
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "ppocrv6-native-server_b200"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def native():
    from ppocr_b200 import capi

    return capi.load()


@pytest.fixture(scope="session")
def oracle_c():
    """The C oracle library (oracle/_build/liboracle.so)."""
    path = REPO / "oracle" / "_build" / "liboracle.so"
    if not path.exists():
        import subprocess

        subprocess.run(["make", "-C", str(REPO / "oracle"), "all"], check=True, capture_output=True)
    lib = ctypes.CDLL(str(path))
    P = ctypes.c_void_p
    lib.oracle_argmax_prob.argtypes = [P, ctypes.c_long, ctypes.c_int, P, P, P, ctypes.c_int]
    lib.oracle_ctc_collapse.argtypes = [P, P, ctypes.c_long, ctypes.c_int, ctypes.c_int, P, P, P]
    return lib


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def parity_report():
    """Measured parity figures (max-abs, relative L2) collected by the tests;
    written as JSON to $PPOCR_PARITY_REPORT at the end of the session when
    that variable is set."""
    import json

    report = {}
    yield report
    path = os.environ.get("PPOCR_PARITY_REPORT")
    if path and report:
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        Path(path).write_text(json.dumps(report, indent=1, sort_keys=True) + "\n")


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream_handle():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
