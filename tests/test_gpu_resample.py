"""Device channel fold and resampling (trc_remix / trc_resample) against their CPU restatements, and the
separator's path for other sample rates and channel counts."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import resample_oracle as RO
from turbo_roformer_b200 import audio
from turbo_roformer_b200 import synthetic as S
from turbo_roformer_b200.resample import design, remix_device, resample_device

from .conftest import snr_db

pytestmark = pytest.mark.gpu

RATES = [(48000, 44100), (44100, 48000), (22050, 44100), (44100, 22050), (96000, 44100), (44100, 32000)]


@pytest.mark.parametrize("sr_in,sr_out", RATES)
@pytest.mark.parametrize("channels,n", [(2, 20011), (1, 5), (3, 1), (6, 4097)])
def test_resample_kernel_matches_oracle(cuda_device, sr_in, sr_out, channels, n):
    """fp64 accumulation on both sides: equal up to the final rounding to float32 (|diff| <= 1 ulp)."""
    f = design(sr_in, sr_out)
    x = np.random.default_rng(n + channels).standard_normal((channels, n)).astype(np.float32)
    got = resample_device(torch.from_numpy(x).to(cuda_device), sr_in, sr_out).cpu().numpy()
    ref = RO.resample(x, f.up, f.down, f.h, f.output_length(n)).astype(np.float32)
    assert got.shape == ref.shape
    tol = np.spacing(np.maximum(np.abs(ref), 1e-30).astype(np.float32)) + 1e-30
    assert (np.abs(got - ref) <= tol).all()


def test_resample_length_trims_and_pads(cuda_device):
    x = torch.from_numpy(np.random.default_rng(0).standard_normal((2, 1000)).astype(np.float32)).to(cuda_device)
    full = resample_device(x, 48000, 44100)
    assert full.shape == (2, 919)
    short = resample_device(x, 48000, 44100, length=500)
    torch.testing.assert_close(short, full[:, :500], rtol=0, atol=0)
    long = resample_device(x, 48000, 44100, length=1000)
    torch.testing.assert_close(long[:, :919], full, rtol=0, atol=0)
    assert not long[:, 919:].any()


@pytest.mark.parametrize("channels", [1, 2, 3, 5, 6, 8, 16])
def test_remix_kernel_matches_to_stereo(cuda_device, channels):
    x = np.random.default_rng(channels).standard_normal((channels, 30001)).astype(np.float32)
    got = remix_device(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(got, audio.to_stereo(x))  # same operations in the same order


@pytest.fixture(scope="module")
def sep(tiny_sd, tiny_cfg, cuda_device):
    from turbo_roformer_b200.separator import Separator

    return Separator.from_module(tiny_sd, tiny_cfg.stft_hop_length, tiny_cfg.dim_t, batch=3)


@pytest.mark.parametrize("sr", [48000, 22050])
def test_separate_other_rate_matches_host_conversion(sep, sr):
    """separate(mix, sr) on the GPU path equals converting with the CPU restatement, separating at
    44.1 kHz and converting back (>= 60 dB: only the resampler's float32 rounding differs)."""
    n = int(1.3 * sr)
    mix = S.chunk_audio(n, seed=31) * np.float32(0.5)
    got = sep.separate(mix, sr=sr)
    assert got.shape == mix.shape and got.dtype == np.float32
    f_in, f_out = design(sr, 44100), design(44100, sr)
    n44 = round(n * 44100 / sr)
    x44 = RO.resample(mix, f_in.up, f_in.down, f_in.h, f_in.output_length(n))[:, :n44].astype(np.float32)
    inst44 = sep.separate(x44)
    ref = RO.resample(inst44, f_out.up, f_out.down, f_out.h, f_out.output_length(n44))[:, :n].astype(np.float32)
    assert snr_db(ref, got) >= 60.0


def test_separate_surround_matches_host_fold(sep):
    """A 5.1 mix separates exactly like its host downmix (the device fold is bit-identical), and the
    centre channel survives the fold on both sides."""
    mix6 = np.random.default_rng(9).standard_normal((6, 40000)).astype(np.float32) * np.float32(0.2)
    np.testing.assert_array_equal(sep.separate(mix6), sep.separate(audio.downmix_stereo(mix6)))
    centre = np.zeros_like(mix6)
    centre[2] = mix6[2]
    folded = remix_device(torch.from_numpy(centre).cuda()).cpu().numpy()
    assert np.abs(folded).max() > 0.2 * np.abs(mix6[2]).max()
    np.testing.assert_array_equal(folded[0], folded[1])


@pytest.mark.parametrize("sr", [48000, 22050, 32000])
def test_other_sample_rates(sep, sr):
    n = int(1.5 * sr)
    mix = S.chunk_audio(n, seed=sr) * np.float32(0.5)
    inst = sep.separate(mix, sr=sr)
    assert inst.shape == (2, n) and inst.dtype == np.float32
    assert np.isfinite(inst).all()


def test_48k_close_to_44k(sep):
    """A 48 kHz copy of a mix separates like the 44.1 kHz original (interior, after converting back)."""
    from turbo_roformer_b200.resample import resample_device

    mix44 = S.chunk_audio(2 * 44100, seed=11) * np.float32(0.5)
    mix48 = resample_device(torch.from_numpy(mix44).cuda(), 44100, 48000).cpu().numpy()
    inst44 = sep.separate(mix44)
    inst48 = sep.separate(mix48, sr=48000)
    back = resample_device(torch.from_numpy(inst48).cuda(), 48000, 44100, length=mix44.shape[1]).cpu().numpy()
    assert snr_db(inst44[:, 2000:-2000], back[:, 2000:-2000]) > 20


def test_separate_other_rate_rejects_nan(sep):
    mix = np.zeros((2, 30000), np.float32)
    mix[0, 100] = np.nan
    with pytest.raises(ValueError):
        sep.separate(mix, sr=48000)
