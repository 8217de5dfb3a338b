"""Chunk schedule and overlap-add: the reference's exact-value pins (tests/test_chunking.py of the reference)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import chunking_oracle as O
from turbo_roformer_b200.chunking import chunk_starts, hamming, overlap_add, step_for


def test_schedule_matches_reference_example(golden_tiny):
    n, chunk = 11130532, 749259
    starts = chunk_starts(n, chunk, step_for(chunk, 2))
    assert step_for(chunk, 2) == 374629
    assert len(starts) == 29
    assert starts[:3] == [0, 374629, 749258]
    assert starts[-1] == n - chunk


def test_song_schedule_matches_golden(golden_tiny):
    n, chunk = 11_130_840, 749_259
    assert chunk_starts(n, chunk, step_for(chunk, 2.0)) == golden_tiny["song_starts"].tolist()


@pytest.mark.parametrize("n", [1, 100, 999, 1000, 1001, 5000, 12345])
@pytest.mark.parametrize("overlap", [1.0, 1.5, 2.0, 3.0])
def test_schedule_covers_signal_and_matches_oracle(n, overlap):
    chunk = 1000
    C = min(chunk, n)
    starts = chunk_starts(n, C, step_for(C, overlap))
    assert starts == O.chunk_starts(n, C, O.step_for(C, overlap))
    covered = np.zeros(n, bool)
    for s in starts:
        assert 0 <= s <= n - C
        covered[s : s + C] = True
    assert covered.all()
    assert starts == sorted(set(starts))


def test_hamming_matches_numpy_and_golden(golden_tiny):
    for n in (1, 2, 7, 1000):
        np.testing.assert_allclose(hamming(n), np.hamming(n), rtol=0, atol=1e-6)
        np.testing.assert_array_equal(hamming(n), O.hamming(n))
    np.testing.assert_array_equal(hamming(1000), golden_tiny["hamming_1000"])
    assert hamming(1000).min() > 0.07


# The overlap-add semantics of the reference's own tests, on the oracle (CPU) ...
@pytest.mark.parametrize("n", [700, 1000, 4321, 10007])
@pytest.mark.parametrize("overlap", [1.0, 1.5, 2.0, 3.0])
def test_identity_model_reconstructs_input(n, overlap):
    x = torch.randn(2, n)
    torch.testing.assert_close(O.overlap_add(x, 1000, overlap, lambda c: c), x, rtol=0, atol=1e-5)


@pytest.mark.parametrize("overlap", [1.5, 2.0, 3.0])
def test_no_click_with_chunk_dependent_model(overlap):
    n, chunk = 100_000, 16000
    x = torch.ones(2, n)
    gains = iter([0.8, 1.2] * 100)
    y = O.overlap_add(x, chunk, overlap, lambda c: c * next(gains)).numpy()
    assert y.min() >= 0.8 - 1e-6 and y.max() <= 1.2 + 1e-6
    assert np.abs(np.diff(y, axis=1)).max() < 0.25 * 0.4
    hard = O.overlap_add(x, chunk, 1.0, lambda c: c * next(gains)).numpy()
    assert np.abs(np.diff(hard, axis=1)).max() > 0.39


def test_overlap_add_has_no_host_path():
    """The package's overlap_add sums on the GPU only: host tensors with a plain callable are refused."""
    with pytest.raises(ValueError):
        overlap_add(torch.randn(2, 5000), 1000, 2.0, lambda c: c)


# ... and the package's device overlap-add against the oracle, bit for bit (same chunk outputs)
@pytest.mark.gpu
@pytest.mark.parametrize("n", [700, 1000, 4321, 10007])
@pytest.mark.parametrize("overlap", [1.0, 1.5, 2.0, 3.0])
def test_device_overlap_add_equals_oracle(cuda_device, n, overlap):
    x = torch.randn(2, n, generator=torch.Generator().manual_seed(n))
    y = overlap_add(x.to(cuda_device), 1000, overlap, lambda c: c)
    assert y.is_cuda
    torch.testing.assert_close(y.cpu(), O.overlap_add(x, 1000, overlap, lambda c: c), rtol=0, atol=0)
    torch.testing.assert_close(y.cpu(), x, rtol=0, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("overlap", [1.0, 1.5, 3.0])
def test_device_overlap_add_chunk_dependent_model_equals_oracle(cuda_device, overlap):
    n, chunk = 100_000, 16000
    x = torch.rand(2, n, generator=torch.Generator().manual_seed(3))
    g1, g2 = iter([0.75, 1.25] * 100), iter([0.75, 1.25] * 100)  # exact products on either device
    y = overlap_add(x.to(cuda_device), chunk, overlap, lambda c: c * next(g1))
    ref = O.overlap_add(x, chunk, overlap, lambda c: c * next(g2))
    torch.testing.assert_close(y.cpu(), ref, rtol=0, atol=0)


@pytest.mark.gpu
def test_device_overlap_add_progress_and_short_outputs(cuda_device):
    calls = []
    x = torch.randn(2, 5000, generator=torch.Generator().manual_seed(4))
    run = lambda c: c[..., :900]  # noqa: E731  (a model that returns fewer samples than the chunk)
    y = overlap_add(x.to(cuda_device), 1000, 2.0, run, progress=lambda k, n: calls.append((k, n)))
    n = len(chunk_starts(5000, 1000, 500))
    assert calls == [(k, n) for k in range(1, n + 1)]
    torch.testing.assert_close(y.cpu(), O.overlap_add(x, 1000, 2.0, run), rtol=0, atol=0)


def test_invalid_schedule_arguments():
    with pytest.raises(ValueError):
        chunk_starts(0, 10, 5)


def test_stream_plan_reproduces_the_schedule():
    """Streaming the schedule over random arrival patterns runs exactly chunk_starts(n) in start order, and
    every chunk of the final schedule that covers a sample reported final has already run."""
    import random

    from turbo_roformer_b200.chunking import chunk_starts, stream_plan

    rnd = random.Random(1)
    for _ in range(5000):
        C = rnd.randint(1, 50)
        step = rnd.randint(1, C)
        n_final = rnd.randint(C, 400)
        cuts = sorted(rnd.sample(range(1, n_final), min(n_final - 1, rnd.randint(0, 10)))) + [n_final]
        full = chunk_starts(n_final, C, step)
        nxt, ran, final_end = 0, [], 0
        for n in cuts:
            st, end = stream_plan(n, nxt, C, step, final=False)
            ran += st
            if st:
                nxt = st[-1] + step
            assert end >= final_end
            final_end = end
            assert all(s in ran for s in full if s < end)
        st, end = stream_plan(n_final, nxt, C, step, final=True)
        ran += st
        assert ran == full and end == n_final
