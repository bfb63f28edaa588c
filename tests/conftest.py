import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device; run the CPU suite with -m 'not gpu'")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ext():
    from laplacianformer_b200.ops import ext as _ext

    return _ext()


@pytest.fixture(scope="session")
def ref_module():
    """The reference operators compiled by oracle/build_ref.py (None if not built)."""
    from oracle.build_ref import load_ref

    return load_ref()
