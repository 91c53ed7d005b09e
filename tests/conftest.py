"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on any host (oracle pinning, host-side pack code, the C ABI surface, gloo ranks);
`-m gpu` needs a B200 and calls the CUDA path through the C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "ork-driver_b200"), os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200; calls the CUDA path through the C ABI")


@pytest.fixture(scope="session")
def ctx():
    import ork_b200

    c = ork_b200.Context()
    yield c
    c.close()


@pytest.fixture
def env_clean(monkeypatch):
    """Pack-time env switches of the reference (ORK_NF4, ORK_SR) unset for the test."""
    monkeypatch.delenv("ORK_NF4", raising=False)
    monkeypatch.delenv("ORK_SR", raising=False)
    return monkeypatch
