"""Shared test setup. `-m gpu` tests need a CUDA device (a B200); everything else runs on the CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "speech.cpp_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu on a B200)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle, build
    build(ref=False)
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle import RefSampler, ref_available
    if not ref_available():
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built here")
    return RefSampler()


@pytest.fixture(scope="session")
def engine():
    """The CUDA engine on cuda:0 (GPU tests only). Fails loudly when the library is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import speech_sampler
    s = speech_sampler.Sampler(0)
    yield s
    s.close()
