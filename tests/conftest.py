"""Test configuration: the `gpu` marker, shared fixtures (seeded synthetic models, the oracle)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def tiny_path():
    from nunchi_b200 import synth
    return synth.cached_gguf("tiny")


@pytest.fixture(scope="session")
def small_path():
    from nunchi_b200 import synth
    return synth.cached_gguf("small")


@pytest.fixture(scope="session")
def wide_path():
    from nunchi_b200 import synth
    return synth.cached_gguf("wide_heads")


@pytest.fixture(scope="session")
def seoul_path():
    from nunchi_b200 import synth
    return synth.cached_gguf("seoul")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """The oracle and the engine library are built in-tree (build() does both); build here if missing."""
    import subprocess
    if not all(os.path.exists(os.path.join(ROOT, "oracle", f)) for f in ("liboracle.so", "liboracle_cr.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)
    yield
