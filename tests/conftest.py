import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qora-tts-12hz-1.7b_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running parity case")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    O.set_threads(8)
    return O


@pytest.fixture(scope="session")
def qtts():
    import qtts_b200
    return qtts_b200


@pytest.fixture(scope="session")
def tiny_path(qtts):
    from qtts_b200 import workload as W
    return W.model_path("tiny")


@pytest.fixture(scope="session")
def p1p7b_path(qtts):
    from qtts_b200 import workload as W
    return W.model_path("1p7b")


@pytest.fixture(scope="session")
def tiny_oracle(oracle_mod, tiny_path):
    m = oracle_mod.Model(tiny_path)
    yield m
    m.close()


@pytest.fixture(scope="session")
def gpu_tiny(qtts, tiny_path):
    if not has_gpu():
        pytest.skip("no GPU")
    m = qtts.Model(tiny_path, 0)
    yield m
    m.close()


@pytest.fixture(scope="session")
def gpu_1p7b(qtts, p1p7b_path):
    if not has_gpu():
        pytest.skip("no GPU")
    m = qtts.Model(p1p7b_path, 0)
    yield m
    m.close()


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False))
