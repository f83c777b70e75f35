import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path through the C ABI")
    # The adjoint-row plugin (libr97host.so) registers its rows into the reference's registry when it is
    # loaded, so the registry (the reference's own host library, loaded RTLD_GLOBAL) goes into this process
    # first: then it does not matter which test -- the optimiser's, the adapter files', the plugin's --
    # loads the plugin first.
    import oracle
    if oracle.ref_available():
        oracle.ref_lib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    return torch.device("cuda", 0)
