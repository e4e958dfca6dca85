"""Shared fixtures.  `-m gpu` tests need a CUDA device and the built library;
everything else runs on the CPU."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")

# Parity tolerance for bf16 decode vs the float32 reference forward
# (north star): |gpu - ref| <= ATOL + RTOL * |ref| elementwise, and greedy
# argmax equal wherever the reference top-2 margin exceeds MARGIN.
ATOL = 3e-2
RTOL = 2e-2
MARGIN = 0.05


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libb2d.so")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


@pytest.fixture(scope="session")
def params306():
    from transformer_b200.config import CONFIG_306M
    from transformer_b200.synth import synth_params
    return synth_params(CONFIG_306M, seed=0)


@pytest.fixture(scope="session")
def params306_f32(params306):
    from transformer_b200.synth import params_f32
    return params_f32(params306)


@pytest.fixture(scope="session")
def params_tiny():
    from transformer_b200.config import CONFIG_TINY
    from transformer_b200.synth import synth_params
    return synth_params(CONFIG_TINY, seed=0)


def _cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    if not _cuda_ok():
        pytest.skip("no CUDA device")
    import torch
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def engine306(cuda, params306):
    from transformer_b200.config import CONFIG_306M
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.packing import prepare_decode_weights_nlayer
    w = prepare_decode_weights_nlayer(params306, CONFIG_306M, device=cuda)
    eng = DecodeEngine(w)
    yield eng
    eng.close()


@pytest.fixture(scope="session")
def engine_tiny(cuda, params_tiny):
    from transformer_b200.config import CONFIG_TINY
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.packing import prepare_decode_weights_nlayer
    w = prepare_decode_weights_nlayer(params_tiny, CONFIG_TINY, device=cuda)
    eng = DecodeEngine(w)
    yield eng
    eng.close()


def assert_logits_close(got, ref, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    bound = ATOL + RTOL * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (f"{what}: {bad.sum()} logits outside atol={ATOL} rtol={RTOL}; "
                           f"max abs err {err.max():.4g}")
    return float(err.max())


@pytest.fixture(scope="session")
def engine306_batched(engine306):
    """The 306M weights bound a second time with a batched workspace."""
    from transformer_b200.multi_sm_decode import DecodeEngine
    eng = DecodeEngine(engine306.w, max_batch=256)
    yield eng
    eng.close()


@pytest.fixture(scope="session")
def engine_tiny_batched(engine_tiny):
    from transformer_b200.multi_sm_decode import DecodeEngine
    eng = DecodeEngine(engine_tiny.w, max_batch=64)
    yield eng
    eng.close()
