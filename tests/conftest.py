import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def ctx():
    """One sulimo context on cuda:0 for the GPU tests (OclContext::new in the reference)."""
    import torch
    import sulimo_b200 as sb
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.init()
    c = sb.CudaContext(0)
    # launch on torch's current stream so torch-side copies and our kernels are ordered
    c.set_stream(torch.cuda.current_stream())
    yield c
    c.close()
