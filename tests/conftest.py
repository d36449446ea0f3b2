import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built plugin")


@pytest.fixture(scope="session")
def port():
    from oracle.oracle import Port, build
    build()
    return Port()


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import REF_LIB, Ref, build
    build()
    if not os.path.exists(REF_LIB):
        pytest.skip("the reference's CPU kernels were not built (no reference checkout here)")
    return Ref()


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def plugin():
    import torch
    from katali_lab_b200 import Plugin
    from katali_lab_b200.build import build
    build()
    assert torch.cuda.is_available(), "GPU test without a GPU"
    p = Plugin()
    assert p.probe(), p.status()
    return p


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch
