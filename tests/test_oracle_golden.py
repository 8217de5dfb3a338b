"""The CPU oracle against the golden vectors produced by the reference implementation itself.

tests/golden/make_golden.py ran the reference package on these seeded weights and inputs; the oracle
must reproduce it (it restates the same fp32 torch math, so agreement is near bit-exact).
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import chunking_oracle, roformer_oracle
from turbo_roformer_b200 import synthetic as S

from .conftest import GOLDEN, snr_db


@pytest.mark.parametrize("name,n,seed", [("chunk", 16256, 0), ("odd5000", 5000, 1), ("odd385", 385, 2)])
def test_oracle_matches_reference_tiny(tiny_cfg, tiny_sd, golden_tiny, name, n, seed):
    x = torch.from_numpy(S.chunk_audio(n, seed=seed)).unsqueeze(0)
    y = roformer_oracle.forward(x, tiny_sd, tiny_cfg)[0].numpy()
    ref = golden_tiny[f"{name}_out"]
    assert y.shape == ref.shape == (2, tiny_cfg.stft_hop_length * (n // tiny_cfg.stft_hop_length))
    assert snr_db(ref, y) >= 110.0


def test_oracle_separate_matches_reference(tiny_cfg, tiny_sd, golden_tiny):
    mix = S.chunk_audio(44100, seed=7) * 3.0
    run = lambda c: roformer_oracle.forward(c, tiny_sd, tiny_cfg)  # noqa: E731
    inst = chunking_oracle.separate_44k(mix, tiny_cfg.chunk, tiny_cfg.stft_hop_length, 2.0, run)
    assert snr_db(golden_tiny["separate_inst"], inst) >= 110.0
    short = chunking_oracle.separate_44k(S.chunk_audio(300, seed=8), tiny_cfg.chunk, tiny_cfg.stft_hop_length, 2.0, run)
    assert short.shape == (2, 300)
    assert snr_db(golden_tiny["separate_short_inst"], short) >= 110.0


def test_golden_metadata_pins_oracle():
    with open(os.path.join(GOLDEN, "golden_meta.json")) as f:
        meta = json.load(f)
    for k in ("tiny_chunk", "tiny_odd5000", "tiny_odd385", "full_chunk", "tiny_separate"):
        assert meta[f"{k}_oracle_snr_db"] >= 120.0


def test_stage_shapes_tiny(tiny_cfg, tiny_sd):
    st: dict = {}
    x = torch.from_numpy(S.chunk_audio(tiny_cfg.chunk, seed=0)).unsqueeze(0)
    roformer_oracle.forward(x, tiny_sd, tiny_cfg, stages=st)
    T = 1 + tiny_cfg.chunk // tiny_cfg.stft_hop_length
    assert st["xin"].shape == (1, T, 4 * tiny_cfg.n_freqs)
    assert st["X0"].shape == (1, T, tiny_cfg.n_bands, 256)
    assert st["mask"].shape == (1, T, 4 * tiny_cfg.n_freqs)


@pytest.mark.slow
def test_oracle_matches_reference_full_chunk_excerpt(full_cfg, full_sd, golden_full):
    """Full-size model, one 17 s chunk (749,700 samples): excerpt, energy and stage excerpts."""
    x = torch.from_numpy(S.chunk_audio(749_700, seed=0)).unsqueeze(0)
    st: dict = {}
    y = roformer_oracle.forward(x, full_sd, full_cfg, stages=st)[0].numpy()
    assert y.shape == (2, 749_700)
    assert snr_db(golden_full["excerpt"], y[:, 300_000:304_096]) >= 100.0
    np.testing.assert_allclose((y.astype(np.float64) ** 2).sum(axis=1), golden_full["sumsq"], rtol=1e-6)
    np.testing.assert_allclose(st["mask"][0, 800:808].numpy(), golden_full["mask_excerpt"], rtol=1e-4, atol=1e-6)
