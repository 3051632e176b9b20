"""pytest setup: the `gpu` marker, import paths, and built libraries.

Tests marked `gpu` need a CUDA device (a B200); everything else runs on the
CPU.  The oracle (oracle/liboracle.so) and the product library
(tensorbit-run_b200/lib/libtb_b200.so) are built on first use if missing.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tensorbit-run_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _ensure_built():
    from oracle import oracle as O
    import tb_b200
    if not os.path.exists(O.PORT_SO):
        O.build()
    if not os.path.exists(tb_b200.LIB_PATH):
        tb_b200.build()


_ensure_built()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
