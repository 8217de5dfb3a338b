"""Host-side audio helpers of the Separator contract (turbo_roformer/audio.py:16-131).

Validation, channel layout and downmix are restated here because ``Separator.separate`` applies them
before the model; resampling (soxr) and file I/O (soundfile) are optional dependencies, imported on use
exactly like the reference does.
"""

from __future__ import annotations

import os

import numpy as np

MAX_CHANNELS = 16


def check_finite(a: np.ndarray) -> None:
    if not np.isfinite(a).all():
        raise ValueError("input contains NaN or inf samples")


def as_channels_first(mix, finite: bool = True) -> np.ndarray:
    """Validate and convert to float32 (channels, samples); raises ValueError like audio.py:16-32.

    ``finite=False`` leaves the NaN/inf scan to the caller (the CUDA separator runs it on the device)."""
    a = np.asarray(mix)
    if a.dtype.kind != "f":
        raise ValueError(f"expected a floating point array (got dtype {a.dtype}); scale integer PCM to [-1, 1] first")
    if a.ndim == 1:
        a = a[None, :]
    elif a.ndim != 2:
        raise ValueError(f"expected (channels, samples) or (samples,), got shape {a.shape}")
    if a.shape[0] > MAX_CHANNELS:
        raise ValueError(f"got {a.shape[0]} channels - is the array (samples, channels)? pass mix.T")
    if a.shape[0] == 0 or a.shape[1] == 0:
        raise ValueError("empty input")
    a = a.astype(np.float32, copy=False)
    if finite:
        check_finite(a)
    return a


def downmix_stereo(x: np.ndarray) -> np.ndarray:
    """(C > 2, n) -> (2, n): centre into both sides at -3 dB, LFE dropped for C >= 6, other channels
    alternately left/right at -3 dB, each side normalised by its summed gains (audio.py:35-59)."""
    c = x.shape[0]
    g = 0.7071
    left = x[0].astype(np.float64)
    right = x[1].astype(np.float64)
    gl = gr = 1.0
    if c >= 3:
        left = left + g * x[2]
        right = right + g * x[2]
        gl += g
        gr += g
    extra = range(4 if c >= 6 else 3, c)
    for k, ch in enumerate(extra):
        if k % 2 == 0:
            left = left + g * x[ch]
            gl += g
        else:
            right = right + g * x[ch]
            gr += g
    return np.stack([left / gl, right / gr]).astype(np.float32)


def to_stereo(x: np.ndarray) -> np.ndarray:
    """Mono duplicated, stereo passed through, more channels downmixed (audio.py:62-68)."""
    if x.shape[0] == 1:
        return np.repeat(x, 2, axis=0)
    if x.shape[0] == 2:
        return np.ascontiguousarray(x)
    return downmix_stereo(x)


def resample(x: np.ndarray, sr_in: int, sr_out: int, length: int | None = None) -> np.ndarray:
    """(C, n) -> (C, m) with soxr HQ; ``length`` forces the output length (audio.py:71-82)."""
    if sr_in != sr_out:
        import soxr  # optional dependency, as in the reference

        y = soxr.resample(np.ascontiguousarray(x.T), sr_in, sr_out, quality="HQ").T
        y = np.asarray(y, dtype=np.float32).reshape(x.shape[0], -1)
    else:
        y = x
    if length is not None and y.shape[1] != length:
        y = y[:, :length] if y.shape[1] > length else np.pad(y, ((0, 0), (0, length - y.shape[1])))
    return np.ascontiguousarray(y, dtype=np.float32)


def load(path: str | os.PathLike) -> tuple[np.ndarray, int]:
    """Read an audio file -> ((channels, samples) float32, sample rate) via soundfile (optional dependency)."""
    import soundfile as sf

    data, sr = sf.read(str(path), dtype="float32", always_2d=True)
    return np.ascontiguousarray(data.T), int(sr)


def output_formats() -> tuple[str, ...]:
    return ("wav", "flac")


def write(path: str | os.PathLike, data: np.ndarray, sr: int, fmt: str = "wav") -> None:
    import soundfile as sf

    subtype = "FLOAT" if fmt == "wav" else "PCM_24"
    sf.write(str(path), np.ascontiguousarray(data.T), sr, subtype=subtype, format=fmt.upper())
