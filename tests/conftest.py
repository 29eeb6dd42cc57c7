"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on the CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; runs the CUDA kernels")


@pytest.fixture(scope="session")
def lz():
    from l0llm_b200 import levelzero

    levelzero.load_library()
    return levelzero


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def device(lz):
    # GPU tests fail (not skip) without a device: the CUDA path is the product, there is no fallback.
    if not lz.LevelZeroRuntime.IsAvailable():
        pytest.fail("no sm_100 device is available for a gpu-marked test")
    d = lz.ComputeDevice(0)
    yield d
    d.Dispose()


@pytest.fixture(scope="session")
def suite(lz, device):
    s = lz.LlmKernelSuite.Create(device)
    yield s
    s.Dispose()
