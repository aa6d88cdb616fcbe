import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the CUDA path")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_lib():
    """The built CUDA library (built in-tree if missing).  No fallback."""
    from tinygpt_b200 import build, _lib
    build.build()
    return _lib.load()


@pytest.fixture(scope="session")
def sampler_factory(cuda_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from tinygpt_b200.sampler import Sampler
    cache = {}

    def make(vocab, max_batch=4096):
        key = (vocab, max_batch)
        if key not in cache:
            cache[key] = Sampler(vocab, max_batch, 0)
        return cache[key]
    return make


# Parity pins report what they exempted (draws near a cumulative boundary,
# probabilities below the mass quantum); the counts are printed at the end of
# the run, visible under -q too.
PIN_REPORT: list[str] = []


@pytest.fixture
def pin_report():
    return PIN_REPORT


def pytest_terminal_summary(terminalreporter):
    if PIN_REPORT:
        terminalreporter.section("parity pin exemptions")
        for line in PIN_REPORT:
            terminalreporter.write_line(line)
