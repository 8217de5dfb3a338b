"""The device resampler's filter and its CPU restatement (no GPU): the oracle equals scipy's polyphase
resampler with the same filter, the filter meets its passband / stopband figures, and the channel fold
restatement equals audio.to_stereo."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import scipy.signal as sg

from oracle import resample_oracle as RO
from turbo_roformer_b200 import _lib, audio
from turbo_roformer_b200.resample import design

RATES = [(48000, 44100), (44100, 48000), (22050, 44100), (44100, 22050), (96000, 44100), (44100, 32000)]


@pytest.mark.parametrize("sr_in,sr_out", RATES)
def test_oracle_equals_scipy_resample_poly(sr_in, sr_out):
    f = design(sr_in, sr_out)
    x = np.random.default_rng(sr_in + sr_out).standard_normal((2, 3001))
    n_out = f.output_length(x.shape[1])
    ref = sg.resample_poly(x, f.up, f.down, axis=1, window=f.h)
    got = RO.resample(x, f.up, f.down, f.h, n_out)
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() < 1e-12


def test_taps_table_is_the_prototype_by_phase():
    f = design(48000, 44100)
    assert (f.up, f.down) == (147, 160) and len(f.h) == 2 * f.half + 1
    flat = f.taps.reshape(-1)
    np.testing.assert_array_equal(flat[: len(f.h)], f.h * f.up)
    assert not flat[len(f.h) :].any()
    np.testing.assert_allclose(f.h, f.h[::-1], atol=0)  # linear phase


@pytest.mark.parametrize("sr_in,sr_out", [(48000, 44100), (44100, 48000), (96000, 44100)])
def test_filter_quality_on_sines(sr_in, sr_out):
    """Passband: a 1 kHz tone and one at 0.9 of the lower Nyquist frequency come out at < -120 dB error
    (interior samples); a tone above the output's Nyquist frequency is suppressed by > 120 dB."""
    f = design(sr_in, sr_out)
    n = sr_in // 2
    t = np.arange(n) / sr_in
    nyq = min(sr_in, sr_out) / 2
    tones = [1000.0, 0.9 * nyq] + ([1.06 * nyq] if sr_out < sr_in else [])
    for hz in tones:
        x = np.sin(2 * np.pi * hz * t)[None]
        y = sg.resample_poly(x, f.up, f.down, axis=1, window=f.h)[0]
        ref = np.sin(2 * np.pi * hz * np.arange(len(y)) / sr_out) if hz < nyq else np.zeros(len(y))
        mid = slice(len(y) // 4, 3 * len(y) // 4)
        err_db = 10 * np.log10(np.mean((y[mid] - ref[mid]) ** 2) / 0.5)
        assert err_db < -120, (hz, err_db)


@pytest.mark.parametrize("channels", [3, 4, 5, 6, 8, 16])
def test_fold_restatement_equals_to_stereo(channels):
    x = np.random.default_rng(channels).standard_normal((channels, 2000)).astype(np.float32)
    np.testing.assert_array_equal(RO.fold(x, audio.stereo_gains(channels)), audio.to_stereo(x))


def test_remix_and_resample_reject_bad_arguments_on_host():
    lib = _lib.load()
    g = (ctypes.c_double * 34)()
    assert lib.trc_remix(ctypes.c_void_p(1), 17, 10, g, ctypes.c_void_p(1), None) == -1
    assert lib.trc_remix(None, 2, 10, g, ctypes.c_void_p(1), None) == -1
    assert lib.trc_resample(ctypes.c_void_p(1), 2, 10, 0, 1, 0, ctypes.c_void_p(1), 4, 10, ctypes.c_void_p(1),
                            None) == -1
    assert lib.trc_resample(ctypes.c_void_p(1), 2, 10, 2, 1, -1, ctypes.c_void_p(1), 4, 10, ctypes.c_void_p(1),
                            None) == -1
    assert b"resample" in lib.trc_last_error()
