import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "midman-ai_b200"
ORACLE = ROOT / "oracle"
for p in (str(PKG), str(ORACLE), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def mm():
    """The ctypes binding of libmidman_gpu.so (built on demand)."""
    import midman_b200
    if not midman_b200.LIB_PATH.exists():
        spec = importlib.util.spec_from_file_location("mm_build", PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    midman_b200.load()
    return midman_b200
