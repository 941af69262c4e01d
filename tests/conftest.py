import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "xingling-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

WEIGHT_CACHE = os.environ.get("XL_WEIGHT_CACHE", "/tmp/xl_weights")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests through the C ABI")


def _gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def built():
    import build as pkg_build

    pkg_build.build()
    import oracle

    oracle.build(ref=None)
    return True


def weight_dir(shape, name: str) -> str:
    import xl_synth

    return xl_synth.write_weight_tree(os.path.join(WEIGHT_CACHE, name), shape)


@pytest.fixture(scope="session")
def tiny_weights():
    import xl_synth

    return weight_dir(xl_synth.TINY, "tiny")


@pytest.fixture(scope="session")
def full_weights():
    import xl_synth

    return weight_dir(xl_synth.FULL, "full")
