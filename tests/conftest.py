import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("sam-3d-objects-ggml_b200", "oracle", "tests"):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 CUDA device and the built libb2q")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def b2q_mod():
    import b2q
    if not os.path.exists(b2q.LIB_PATH):
        b2q.build()
    return b2q


@pytest.fixture(scope="session")
def dev():
    import torch
    assert torch.cuda.is_available()
    cap = torch.cuda.get_device_capability(0)
    assert cap == (10, 0), f"needs sm_100 (B200), got {cap}"
    return torch.device("cuda:0")
