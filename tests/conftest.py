import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _gpu_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def ctx():
    if not _gpu_present():
        pytest.skip("no CUDA device on this host")
    import flight4s_b200 as f4s
    c = f4s.CudaContext.open(0)
    assert c.compute_capability == (10, 0), f"expected a B200 (sm_100), got {c.compute_capability}"
    yield c
    c.close()


@pytest.fixture(scope="session")
def hp(ctx):
    return ctx.hotpath()


@pytest.fixture(scope="session")
def torch_dev(ctx):
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
