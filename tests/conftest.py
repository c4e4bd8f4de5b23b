"""Shared pytest setup: the `gpu` marker, import paths and library fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "tensorbit-core_b200", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def port():
    from oracle import Oracle
    return Oracle("port")


@pytest.fixture(scope="session")
def ref():
    from oracle import Oracle, ref_available
    if not ref_available():
        pytest.skip("reference oracle not built here (needs the reference sources)")
    return Oracle("ref")


@pytest.fixture(scope="session")
def tblib():
    """The CUDA library, built in-tree if missing (nvcc is part of the image)."""
    import tbabi
    if not os.path.exists(tbabi.LIB_PATH):
        import build
        build.build()
    return tbabi


@pytest.fixture(scope="session")
def cuda(tblib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.init()
    return torch
