"""Seeded synthetic weights and audio for tests and benchmarks (no network: no checkpoints, no datasets).

* ``init_weights`` draws a random-init ``state_dict`` with upstream keys: norm gains 1 + s_g * N(0,1),
  every other weight and bias s_w * N(0,1) ("init A": s_g = s_w = 0.02). Rotary frequencies follow
  the reference formula (turbo_roformer/model.py:42-44).
* ``chunk_audio`` is the single-chunk input (Gaussian noise sigma 0.1 plus three random sines).
* ``song_audio`` is the 252.4 s song (seeded pink noise plus random sine chords).
"""

from __future__ import annotations

import math
from collections import OrderedDict

import numpy as np
import torch

from .config import ModelConfig, param_shapes

SR = 44100


def rotary_freqs(dim_head: int, theta: float = 10000.0) -> torch.Tensor:
    """fp32 rotary frequencies exactly as the reference builds them (model.py:42-44)."""
    return 1.0 / (theta ** (torch.arange(0, dim_head, 2)[: dim_head // 2].float() / dim_head))


def init_weights(
    cfg: ModelConfig, seed: int = 0, gamma_std: float = 0.02, weight_std: float = 0.02, bias_std: float | None = None
) -> "OrderedDict[str, torch.Tensor]":
    """Random-init fp32 state dict (CPU) with the upstream keys and shapes."""
    bias_std = weight_std if bias_std is None else bias_std
    g = torch.Generator().manual_seed(seed)
    out: OrderedDict[str, torch.Tensor] = OrderedDict()
    freqs = rotary_freqs(cfg.dim_head)
    for name, shape in param_shapes(cfg).items():
        if name.endswith("rotary_embed.freqs"):
            out[name] = freqs.clone()
        elif name.endswith("gamma"):
            out[name] = 1.0 + gamma_std * torch.randn(shape, generator=g)
        elif name.endswith("bias"):
            out[name] = bias_std * torch.randn(shape, generator=g)
        else:
            out[name] = weight_std * torch.randn(shape, generator=g)
    return out


def tiny_weights(cfg: ModelConfig, seed: int = 0) -> "OrderedDict[str, torch.Tensor]":
    """Weights for the small test model: non-trivial gains (so folding is exercised) and biases,
    weights at the scale of PyTorch's default Linear init for fan-in 256 (tests/conftest.py:49-58)."""
    return init_weights(cfg, seed=seed, gamma_std=0.25, weight_std=0.036, bias_std=0.05)


def chunk_audio(n: int, seed: int = 0) -> np.ndarray:
    """(2, n) float32: 0.1 * N(0,1) + 3 sines with f ~ U[50, 8000] Hz, a ~ U[0.05, 0.2], random phase."""
    rng = np.random.default_rng(seed)
    x = 0.1 * rng.standard_normal((2, n))
    t = np.arange(n) / SR
    for _ in range(3):
        f = rng.uniform(50.0, 8000.0)
        a = rng.uniform(0.05, 0.2)
        ph = rng.uniform(0.0, 2 * math.pi)
        x += a * np.sin(2 * math.pi * f * t + ph)
    return x.astype(np.float32)


def song_audio(seconds: float = 252.4, seed: int = 0) -> np.ndarray:
    """(2, n) float32 song: pink noise (1/f power) plus random three-note sine chords every 0.5 s."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * SR))
    spec = rng.standard_normal((2, n // 2 + 1)) + 1j * rng.standard_normal((2, n // 2 + 1))
    f = np.fft.rfftfreq(n, 1.0 / SR)
    spec[:, 1:] /= np.sqrt(f[1:])
    spec[:, 0] = 0.0
    pink = np.fft.irfft(spec, n=n, axis=1)
    pink *= 0.1 / pink.std()
    out = pink
    hop = SR // 2
    t = np.arange(2 * hop) / SR
    for start in range(0, n, hop):
        seg = slice(start, min(n, start + 2 * hop))
        m = seg.stop - seg.start
        root = 110.0 * 2 ** (rng.integers(0, 36) / 12)
        env = np.exp(-t[:m] * rng.uniform(1.5, 5.0))
        chord = sum(np.sin(2 * math.pi * root * r * t[:m] + rng.uniform(0, 6.3)) for r in (1.0, 1.26, 1.5))
        pan = rng.uniform(0.2, 0.8)
        out[0, seg] += 0.1 * (1 - pan) * chord * env
        out[1, seg] += 0.1 * pan * chord * env
    out *= 0.8 / np.abs(out).max()
    return out.astype(np.float32)


def service_songs(n_songs: int = 8, seconds: float = 120.0, seed: int = 100) -> list[np.ndarray]:
    """Eight seeded 2-minute songs for the batched service load."""
    return [song_audio(seconds, seed=seed + i) for i in range(n_songs)]


def snr_db(ref, est) -> float:
    """10 log10(|ref|^2 / |ref - est|^2) in float64 (tests/conftest.py:97-100)."""
    ref = np.asarray(ref, np.float64)
    est = np.asarray(est, np.float64)
    return float(10 * np.log10((ref**2).sum() / max(((ref - est) ** 2).sum(), 1e-300)))
