import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "stochastic-rounding-pytorch_b200", ROOT / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU and libsrs_b200.so")
    config.addinivalue_line("markers", "statistical: randomized statistical test")


@pytest.fixture
def fake_launcher(monkeypatch):
    """Route every kernel launch to the CPU oracle (host-logic tests without a GPU)."""
    from _support import FakeLauncher
    from sr_states.cuda import _native

    fake = FakeLauncher()
    previous = _native.set_launcher(fake)
    yield fake
    _native.set_launcher(previous)


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device (run them on a B200)")
    from sr_states.cuda import _native

    _native.launcher().check_device(torch.device("cuda", torch.cuda.current_device()))
    return torch.device("cuda", torch.cuda.current_device())
