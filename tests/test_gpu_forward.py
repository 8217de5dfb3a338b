"""End-to-end parity of the CUDA forward against the reference's fp32 forward (golden vectors / oracle).

The bar is the north star's: >= 50 dB SNR against the fp32 reference on the same weights and audio
(the reference's own bf16 AVX-512 kernels reach 45.5 dB on the small model and 46.8 dB on the full
model with these weights, tests/golden/golden_meta.json).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import roformer_oracle as R
from turbo_roformer_b200 import synthetic as S

from .conftest import snr_db

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,n,seed", [("chunk", 16256, 0), ("odd5000", 5000, 1), ("odd385", 385, 2)])
def test_tiny_forward_matches_reference(tiny_cuda, golden_tiny, name, n, seed):
    x = torch.from_numpy(S.chunk_audio(n, seed=seed)).unsqueeze(0)
    y = tiny_cuda.forward(x)
    ref = golden_tiny[f"{name}_out"]
    assert y.shape == (1,) + ref.shape
    assert y.device.type == "cpu"
    assert snr_db(ref, y[0].numpy()) >= 50.0


def test_batched_forward_equals_single(tiny_cuda, tiny_cfg):
    xs = [S.chunk_audio(tiny_cfg.chunk, seed=s) for s in (11, 12, 13)]
    batch = torch.from_numpy(np.stack(xs)).cuda()
    yb = tiny_cuda.forward_device(batch)
    for i, x in enumerate(xs):
        y1 = tiny_cuda.forward_device(torch.from_numpy(x).unsqueeze(0).cuda())
        torch.testing.assert_close(yb[i : i + 1], y1, rtol=0, atol=0)


def test_forward_is_deterministic(tiny_cuda, tiny_cfg):
    x = torch.from_numpy(S.chunk_audio(tiny_cfg.chunk, seed=21)).unsqueeze(0).cuda()
    a = tiny_cuda.forward_device(x).clone()
    b = tiny_cuda.forward_device(x)
    assert torch.equal(a, b)


def test_bf16_operands_path(tiny_sd, tiny_cfg, golden_tiny, cuda_device):
    from turbo_roformer_b200.backend import CudaBSRoformer

    m = CudaBSRoformer(tiny_sd, cfg=tiny_cfg, device=0, precision="bf16")
    y = m(torch.from_numpy(S.chunk_audio(16256, seed=0)).unsqueeze(0))
    assert snr_db(golden_tiny["chunk_out"], y[0].numpy()) >= 35.0  # bf16 rounding: the reference gets 45.5 dB


def test_rejects_bad_shapes(tiny_cuda):
    with pytest.raises(ValueError):
        tiny_cuda(torch.zeros(1, 1, 1000))
    with pytest.raises(ValueError):
        tiny_cuda(torch.zeros(1, 2, 100))  # not more than n_fft / 2 samples


@pytest.fixture(scope="module")
def full_chunk_ref(full_cfg, full_sd, golden_full):
    """Config 1 input (one 749,700-sample chunk) and the fp32 oracle's output for it."""
    x = torch.from_numpy(S.chunk_audio(749_700, seed=0)).unsqueeze(0)
    ref = R.forward(x, full_sd, full_cfg)[0].numpy()
    # the oracle run here is the one pinned by the reference's own output
    assert snr_db(golden_full["excerpt"], ref[:, 300_000:304_096]) >= 100.0
    return x, ref


@pytest.mark.slow
def test_full_chunk_matches_fp32_reference(full_cfg, full_sd, full_chunk_ref, cuda_device):
    """Config 1: one 17 s chunk (749,700 samples) through the full 12-layer model, >= 50 dB."""
    from turbo_roformer_b200.backend import CudaBSRoformer

    x, ref = full_chunk_ref
    m = CudaBSRoformer(full_sd, cfg=full_cfg, device=0, precision="fp16")
    y = m(x)[0].numpy()
    snr = snr_db(ref, y)
    print(f"config 1, fp16 operands: {snr:.2f} dB vs the fp32 reference forward")
    assert snr >= 50.0


@pytest.mark.slow
def test_full_chunk_bf16_operands(full_cfg, full_sd, full_chunk_ref, cuda_device):
    """Config 1 with bf16 tensor-core operands (the north star's operand type). At these random-init
    weights bf16 rounding alone costs the reference's own bf16 kernels their 50 dB (46.8 dB,
    golden_meta.json); the number is recorded, and held to the reference's band minus 3 dB."""
    from turbo_roformer_b200.backend import CudaBSRoformer

    x, ref = full_chunk_ref
    m = CudaBSRoformer(full_sd, cfg=full_cfg, device=0, precision="bf16")
    y = m(x)[0].numpy()
    snr = snr_db(ref, y)
    print(f"config 1, bf16 operands: {snr:.2f} dB vs the fp32 reference forward")
    assert snr >= 43.8


@pytest.mark.slow
def test_full_model_batch4_equals_single_chunks(full_cfg, full_sd, cuda_device):
    """The bench's shape (four Separator chunks per forward through the full model) is clean and
    bit-identical to one chunk per forward, repeated: the persistent kernels walk ~90 work items per CTA
    here, where a pipeline that lets one query tile run an item ahead would surface."""
    from turbo_roformer_b200.backend import CudaBSRoformer

    m = CudaBSRoformer(full_sd, cfg=full_cfg, device=0, precision="fp16")
    C = 749_259
    song = torch.from_numpy(S.song_audio(4 * C / 44100 + 0.1, seed=3)).cuda()
    frames = torch.stack([song[:, k * C : (k + 1) * C] for k in range(4)]).contiguous()
    singles = torch.cat([m.forward_device(frames[k : k + 1]) for k in range(4)])
    for _ in range(3):
        y = m.forward_device(frames)  # checks the device error word
        assert torch.isfinite(y).all()
        assert torch.equal(y, singles)


def test_bounded_wait_reports_and_recovers(tiny_cuda, tiny_cfg):
    """A pipeline wait that can never complete ends with TRC_E_DEVICE after the wait limit, not a hang or
    a fault, and the handle keeps working (the failure path of every pipelined kernel)."""
    from turbo_roformer_b200 import _lib

    st = ctypes.c_void_p(tiny_cuda.stream_ptr())
    _lib.check(tiny_cuda.lib.trc_selftest_wait_timeout(tiny_cuda.handle, st))
    with pytest.raises(_lib.TRCError, match="device error"):
        tiny_cuda.check()
    x = torch.from_numpy(S.chunk_audio(tiny_cfg.stft_hop_length * 40, seed=3)).unsqueeze(0)
    y = tiny_cuda.forward(x)
    tiny_cuda.check()
    assert torch.isfinite(y).all()
