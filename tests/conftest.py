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


def quantize_edge_data(rng, k=8, n=96):
    """f32 [k][n] rows mixing ordinary weights with every case
    quantize_f32_to_q4 (gemv.rs:92-130) treats specially: all-zero groups,
    exact .5 ties (absmax 7 -> scale 1), NaN and inf inside groups, an
    all-NaN group, subnormal groups, scales that overflow f16, signed zeros."""
    d = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    g = d.reshape(-1, 32)  # view: one row per group
    g[0] = 0.0
    g[1] = np.array([0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 3.5, -3.5, 4.5, -4.5, 5.5, -5.5, 6.5, -6.5, 7.0, -7.0,
                     0.0, -0.0, 1.0, -1.0, 2.0, -2.0, 3.0, -3.0, 0.25, -0.25, 0.75, -0.75, 6.9, -6.9, 0.49, -0.51],
                    np.float32)
    g[2, 3] = np.nan
    g[3] = np.nan
    g[4, 7] = np.inf
    g[5, 0] = -np.inf
    g[6] = (rng.standard_normal(32) * 1e-40).astype(np.float32)  # subnormal f32 scale
    g[7] = (rng.standard_normal(32) * 1e6).astype(np.float32)    # scale beyond f16 range -> inf
    g[8] = -0.0
    g[9] = (rng.standard_normal(32) * 6e-5).astype(np.float32)   # f16-subnormal scales
    g[10, :] = 65504.0 * 7.0                                       # scale at the f16 maximum
    return d


def quantize_np(data):
    """Independent numpy restatement of quantize_f32_to_q4 (gemv.rs:92-130)."""
    g = np.ascontiguousarray(data, np.float32).reshape(-1, 32)
    a = np.abs(g)
    absmax = np.where(np.isnan(a), np.float32(0), a).max(axis=1)  # `v > absmax` never picks NaN
    scale = (absmax / np.float32(7)).astype(np.float32)
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        sh = scale.astype(np.float16).view(np.uint16)
        inv = np.where(scale > 0, np.float32(1) / scale, np.float32(0)).astype(np.float32)
        prod = (g * inv[:, None]).astype(np.float32)
        p64 = prod.astype(np.float64)
        r = np.sign(p64) * np.floor(np.abs(p64) + 0.5)  # round half away from zero (exact in f64)
    r = np.clip(r, -8, 7)
    q = np.where(np.isnan(r), 0, r + 8).astype(np.uint8)  # Rust `NaN as u8` == 0
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    return packed, sh.reshape(-1)
