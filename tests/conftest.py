import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: config-scale case (seconds of GPU time)")


def _build_once():
    """Builds the oracle (and the reference library where the reference tree exists) and the
    C-ABI library if they are missing; on the GPU box both arrive prebuilt."""
    from oracle import build as oracle_build

    if not (REPO / "oracle" / "liboracle.so").exists():
        oracle_build.build_port()
    from matrix_b200 import build as lib_build

    if not lib_build.LIB.exists():
        lib_build.build()


_build_once()


@pytest.fixture(scope="session")
def port():
    from oracle import oracle

    p = oracle.port()
    # every thread runs the reference's scalar loop on its own slice of outputs
    p.threads = int(os.environ.get("ORACLE_THREADS", str(min(32, os.cpu_count() or 1))))
    return p


@pytest.fixture(scope="session")
def ref():
    from oracle import oracle

    r = oracle.reference()
    if r is None:
        pytest.skip("oracle/_ref/libmtx_ref.so not built (reference tree absent when building)")
    return r


@pytest.fixture(scope="session")
def gpu():
    """Initialises the backend on cuda:0 with torch's current stream."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from matrix_b200 import backend

    torch.cuda.set_device(0)
    backend.init(0)
    yield backend
    torch.cuda.synchronize()
