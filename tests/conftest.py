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


@pytest.fixture
def tune(ctx, monkeypatch):
    """tune(name, value): sets one ORKB_* kernel-choice variable for this test and has the session
    context take it (the library reads its tuning variables once per context: ork_b200_reload_tuning).
    Afterwards every ORKB_* variable is cleared and the context re-reads the clean environment."""
    import ork_b200

    L = ork_b200.lib()

    def set_(name, value):
        assert name.startswith("ORKB_")
        monkeypatch.setenv(name, str(value))
        assert L.ork_b200_reload_tuning(ctx.ctx) == 0

    yield set_
    for k in [k for k in os.environ if k.startswith("ORKB_")]:
        monkeypatch.delenv(k)
    L.ork_b200_reload_tuning(ctx.ctx)
