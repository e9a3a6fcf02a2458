"""Shared pytest set-up: the gpu marker, import paths and cached fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "moss-transcribe.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def fixture_dir(tmp_path_factory):
    d = os.environ.get("MTB_FIXTURE_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        return d
    return str(tmp_path_factory.mktemp("gguf"))


@pytest.fixture(scope="session")
def tiny_gguf(fixture_dir):
    from mtb import fixture
    return fixture.cached_fixture(fixture.TINY, seed=0, directory=fixture_dir, parity=True)


@pytest.fixture(scope="session")
def tiny_bench_gguf(fixture_dir):
    from mtb import fixture
    return fixture.cached_fixture(fixture.TINY, seed=0, directory=fixture_dir, parity=False)


@pytest.fixture(scope="session")
def tiny_f16_gguf(fixture_dir):
    """The tiny parity model with F16 weights (token_embd and projections)."""
    from mtb import fixture
    return fixture.cached_fixture(fixture.TINY, seed=0, directory=fixture_dir, parity=True, dtype="f16")


@pytest.fixture(scope="session")
def tiny_f16_oracle(tiny_f16_gguf):
    import oracle
    return oracle.OracleModel(tiny_f16_gguf)


@pytest.fixture(scope="session")
def tiny_oracle(tiny_gguf):
    import oracle
    return oracle.OracleModel(tiny_gguf)
