"""What ``Separator`` does to a mix before the model and to the result after it, on the host.

The separator contract (turbo_roformer/separator.py:203-283, its input rules in turbo_roformer/audio.py):
float input of shape (channels, samples) or (samples,); integer PCM, NaN/inf, empty arrays and arrays
that look transposed are refused with ``ValueError``; mono is played on both sides, more than two
channels are folded to stereo, and rates other than 44.1 kHz are resampled around the model.

Channel handling here is one linear map: a (2, C) gain matrix per channel count, applied in float64.
The fold of a surround layout sends the centre (channel 2) to both sides at -3 dB, drops the LFE
(channel 3) of 5.1 and wider layouts, spreads the remaining channels alternately left and right at
-3 dB, and scales each output side by the inverse of its total gain. Resampling (``soxr``) and file
I/O (``soundfile``) are optional dependencies that are imported only when a call needs them.
"""

from __future__ import annotations

import os
from functools import lru_cache

import numpy as np

MAX_CHANNELS = 16
SIDE_GAIN = 0.7071  # -3 dB
FORMATS = {"wav": "FLOAT", "flac": "PCM_24"}  # output container -> sample encoding


def check_finite(a: np.ndarray) -> None:
    if not np.isfinite(a).all():
        raise ValueError("input contains NaN or inf samples")


def as_channels_first(mix, finite: bool = True) -> np.ndarray:
    """The mix as a float32 (channels, samples) array; ``ValueError`` for input the separator refuses.

    ``finite=False`` skips the NaN/inf scan (the CUDA separator makes it on the device instead)."""
    a = np.asarray(mix)
    if a.dtype.kind != "f":
        raise ValueError(f"expected floating point samples, got dtype {a.dtype} (scale integer PCM to [-1, 1])")
    if a.ndim not in (1, 2):
        raise ValueError(f"expected (channels, samples) or (samples,), got shape {a.shape}")
    a = a.reshape(1, -1) if a.ndim == 1 else a
    channels, samples = a.shape
    if channels > MAX_CHANNELS:
        raise ValueError(f"{channels} channels: the array looks like (samples, channels); pass mix.T")
    if channels * samples == 0:
        raise ValueError("empty input")
    a = np.asarray(a, dtype=np.float32)
    if finite:
        check_finite(a)
    return a


@lru_cache(maxsize=MAX_CHANNELS)
def stereo_gains(channels: int) -> np.ndarray:
    """(2, channels) float64 matrix that maps a layout of ``channels`` channels to (left, right)."""
    if channels < 1:
        raise ValueError("need at least one channel")
    if channels == 1:
        return np.ones((2, 1))
    m = np.zeros((2, channels))
    m[0, 0] = m[1, 1] = 1.0
    if channels >= 3:
        m[:, 2] = SIDE_GAIN
    first_extra = 4 if channels >= 6 else 3  # skip the LFE of 5.1 and wider
    for k, ch in enumerate(range(first_extra, channels)):
        m[k % 2, ch] = SIDE_GAIN
    m /= m.sum(axis=1, keepdims=True)
    m.setflags(write=False)
    return m


def to_stereo(x: np.ndarray) -> np.ndarray:
    """(C, n) float32 -> (2, n) float32 through ``stereo_gains(C)``; stereo input is passed through."""
    if x.shape[0] == 2:
        return np.ascontiguousarray(x, dtype=np.float32)
    if x.shape[0] == 1:
        return np.ascontiguousarray(np.broadcast_to(x, (2, x.shape[1])), dtype=np.float32)
    # channel order, separately rounded products and sums in float64: the device fold (trc_remix) makes
    # the same operations, so both give the same float32 result
    g = stereo_gains(x.shape[0])
    y = np.zeros((2, x.shape[1]))
    for k in range(x.shape[0]):
        y += g[:, k : k + 1] * x[k].astype(np.float64)
    return y.astype(np.float32)


def downmix_stereo(x: np.ndarray) -> np.ndarray:
    """Fold of a layout with more than two channels (kept as a name for callers of the reference API)."""
    if x.shape[0] <= 2:
        raise ValueError("downmix needs more than two channels")
    return to_stereo(x)


def resample(x: np.ndarray, sr_in: int, sr_out: int, length: int | None = None) -> np.ndarray:
    """(C, n) at ``sr_in`` -> (C, m) at ``sr_out`` (soxr, high quality); ``length`` trims or zero-pads
    the result to exactly that many samples."""
    y = np.asarray(x, dtype=np.float32)
    if sr_in != sr_out:
        try:
            import soxr
        except ImportError as e:  # pragma: no cover - depends on the environment
            raise ImportError(f"resampling {sr_in} Hz -> {sr_out} Hz needs the optional package 'soxr'") from e
        y = np.asarray(soxr.resample(np.ascontiguousarray(y.T), sr_in, sr_out, quality="HQ"), dtype=np.float32)
        y = y.reshape(-1, x.shape[0]).T
    if length is not None:
        m = y.shape[1]
        y = y[:, :length] if m >= length else np.concatenate([y, np.zeros((y.shape[0], length - m), np.float32)], 1)
    return np.ascontiguousarray(y, dtype=np.float32)


def output_formats() -> tuple[str, ...]:
    return tuple(FORMATS)


def load(path: str | os.PathLike) -> tuple[np.ndarray, int]:
    """Decode an audio file into (float32 (channels, samples), sample rate); needs 'soundfile'."""
    import soundfile

    frames, sr = soundfile.read(os.fspath(path), dtype="float32", always_2d=True)
    return np.ascontiguousarray(frames.T), int(sr)


def write(path: str | os.PathLike, data: np.ndarray, sr: int, fmt: str = "wav") -> None:
    """Encode (channels, samples) float32 as ``fmt`` (float WAV or 24-bit FLAC); needs 'soundfile'."""
    import soundfile

    if fmt not in FORMATS:
        raise ValueError(f"unsupported output format {fmt!r}")
    soundfile.write(os.fspath(path), np.ascontiguousarray(data.T), sr, subtype=FORMATS[fmt], format=fmt.upper())
