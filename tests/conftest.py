"""Shared fixtures: the small test model, golden fixtures, and the CUDA model (GPU tests only).

Markers: ``gpu`` (needs a B200 and libtrcuda.so), ``slow`` (tens of seconds of CPU oracle work).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

from turbo_roformer_b200 import config as C  # noqa: E402
from turbo_roformer_b200 import synthetic as S  # noqa: E402

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and libtrcuda.so")
    config.addinivalue_line("markers", "slow: runs the full-size CPU oracle")


def snr_db(ref, est) -> float:
    return S.snr_db(ref, est)


@pytest.fixture(scope="session")
def tiny_cfg() -> C.ModelConfig:
    return C.TINY


@pytest.fixture(scope="session")
def tiny_sd(tiny_cfg):
    return S.tiny_weights(tiny_cfg, seed=0)


@pytest.fixture(scope="session")
def golden_tiny():
    return dict(np.load(os.path.join(GOLDEN, "tiny_model.npz")))


@pytest.fixture(scope="session")
def golden_full():
    return dict(np.load(os.path.join(GOLDEN, "full_chunk.npz")))


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def lib(cuda_device):
    from turbo_roformer_b200 import _lib

    return _lib.load(build_if_missing=False)


@pytest.fixture(scope="session")
def tiny_cuda(cuda_device, tiny_sd, tiny_cfg):
    from turbo_roformer_b200.backend import CudaBSRoformer

    return CudaBSRoformer(tiny_sd, cfg=tiny_cfg, device=0, precision="fp16")


@pytest.fixture(scope="session")
def full_cfg() -> C.ModelConfig:
    return C.RESURRECTION


@pytest.fixture(scope="session")
def full_sd(full_cfg):
    return S.init_weights(full_cfg, seed=0)
