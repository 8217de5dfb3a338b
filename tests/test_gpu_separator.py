"""Separator API on the CUDA backend (the reference's tests/test_separator.py cases that need no sound
files; the other-rate and surround cases are in test_gpu_resample.py), checked against the reference's own
Separator output on the small model."""

from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

from oracle import chunking_oracle, roformer_oracle
from turbo_roformer_b200 import synthetic as S

from .conftest import snr_db

pytestmark = pytest.mark.gpu

SR = 44100


@pytest.fixture(scope="module")
def sep(tiny_sd, tiny_cfg, cuda_device):
    from turbo_roformer_b200.separator import Separator

    return Separator.from_module(tiny_sd, tiny_cfg.stft_hop_length, tiny_cfg.dim_t, batch=3)


def test_separate_matches_reference_separator(sep, golden_tiny):
    mix = S.chunk_audio(44100, seed=7) * 3.0  # peak gain path
    inst = sep.separate(mix, overlap=2.0)
    assert inst.shape == mix.shape and inst.dtype == np.float32
    assert snr_db(golden_tiny["separate_inst"], inst) >= 50.0


def test_short_clip_matches_reference(sep, golden_tiny):
    inst = sep.separate(S.chunk_audio(300, seed=8))
    assert inst.shape == (2, 300)
    assert snr_db(golden_tiny["separate_short_inst"], inst) >= 50.0


def test_device_overlap_add_is_bit_identical_to_reference_loop(sep, tiny_cfg):
    """Same chunk outputs -> the device overlap-add equals the reference's sequential loop exactly."""
    from turbo_roformer_b200.chunking import chunk_starts, ola_device, step_for

    mix = S.chunk_audio(3 * SR, seed=5)
    xp, _ = sep.prepare_44k(mix)
    x = torch.from_numpy(xp).cuda()
    C = sep.chunk
    starts = chunk_starts(x.shape[1], C, step_for(C, 2.0))
    ys = sep.net.forward_device(torch.stack([x[:, s : s + C] for s in starts]))
    dev = ola_device(ys, starts, C, x.shape[1]).cpu()
    ref = chunking_oracle.ola_from_outputs(list(ys.cpu()), starts, x.shape[1], C)
    assert torch.equal(dev, ref)


@pytest.mark.parametrize("n", [1, 2, 127, 128, 383, 385, 16255, 16256, 16257])
def test_short_and_boundary_lengths(sep, n):
    mix = S.chunk_audio(max(n, 2), seed=n)[:, :n]
    inst = sep.separate(mix)
    assert inst.shape == (2, n)
    assert np.isfinite(inst).all()


def test_deterministic_and_mono(sep):
    mix = S.chunk_audio(SR, seed=4)
    np.testing.assert_array_equal(sep.separate(mix), sep.separate(mix))
    mono = mix[:1]
    a = sep.separate(mono[0])
    np.testing.assert_array_equal(a, sep.separate(mono))
    np.testing.assert_array_equal(a, sep.separate(np.repeat(mono, 2, axis=0)))


def test_peak_normalisation_is_scale_invariant(sep):
    mix = S.chunk_audio(SR, seed=12)
    a = sep.separate(mix * 2.0) / 2.0
    b = sep.separate(mix * 4.0) / 4.0
    assert snr_db(a, b) > 100


@pytest.mark.parametrize("overlap", [1.0, 1.5, 3.0])
def test_overlaps_match_oracle(sep, tiny_sd, tiny_cfg, overlap):
    mix = S.chunk_audio(SR, seed=13)
    inst = sep.separate(mix, overlap=overlap)
    ref = chunking_oracle.separate_44k(mix, sep.chunk, sep.hop, overlap,
                                       lambda c: roformer_oracle.forward(c, tiny_sd, tiny_cfg))
    assert snr_db(ref, inst) >= 50.0


def test_progress_and_invalid_arguments(sep):
    mix = S.chunk_audio(SR)
    calls = []
    sep.separate(mix, progress=lambda k, n: calls.append((k, n)))
    n = sep.n_chunks(SR)
    assert calls[-1] == (n, n) and all(b == n for _, b in calls)
    with pytest.raises(ValueError):
        sep.separate(mix, overlap=0.5)
    with pytest.raises(ValueError):
        sep.separate(mix, sr=0)
    with pytest.raises(ValueError):
        sep.separate(np.zeros((2, 10), np.int16))
    # the NaN/inf scan runs on the device: the call still raises and the handle stays usable
    for bad in (np.nan, np.inf, -np.inf):
        m = mix.copy()
        m[1, 1234] = bad
        with pytest.raises(ValueError):
            sep.separate(m)
    np.testing.assert_array_equal(sep.separate(mix), sep.separate(mix))


def test_concurrent_calls_are_serialised(sep):
    mix = S.chunk_audio(SR, seed=14)
    expected = sep.separate(mix)
    results = [None] * 3

    def work(i):
        results[i] = sep.separate(mix)

    ts = [threading.Thread(target=work, args=(i,)) for i in range(3)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for r in results:
        np.testing.assert_array_equal(r, expected)


def test_vocals_identity(sep):
    mix = S.chunk_audio(3 * SR, seed=9)
    inst = sep.separate(mix)
    np.testing.assert_allclose(inst + (mix - inst), mix, atol=1e-6)


def test_submit_queues_songs_and_matches_separate(sep):
    songs = [S.chunk_audio(SR * 3 + 77 * k, seed=10 + k) for k in range(3)]
    ref = [sep.separate(m) for m in songs]
    pinned = torch.from_numpy(songs[0]).pin_memory()
    jobs = [sep.submit(pinned)] + [sep.submit(m) for m in songs[1:]]
    # results in reverse order: each job owns its buffers
    got = [j.result() for j in reversed(jobs)][::-1]
    for r, g in zip(ref, got):
        np.testing.assert_array_equal(r, g)
    assert all(j.done() for j in jobs)
    out = torch.empty(2, songs[1].shape[1], dtype=torch.float32).pin_memory()
    np.testing.assert_array_equal(sep.submit(songs[1], out=out).result(), ref[1])
    with pytest.raises(ValueError):
        sep.submit(songs[1], out=torch.empty(2, 5, dtype=torch.float32).pin_memory())
    bad = songs[2].copy()
    bad[0, 99] = np.nan
    job = sep.submit(bad)
    with pytest.raises(ValueError):
        job.result()
    np.testing.assert_array_equal(sep.submit(songs[2]).result(), ref[2])  # the handle stays usable


def test_submit_mono_and_surround_equal_separate(sep):
    """Mono and 5.1 mixes queued with submit (folded on the GPU) equal separate() of the same mixes."""
    mono = S.chunk_audio(SR * 2, seed=31)[0]
    six = (np.random.default_rng(32).standard_normal((6, SR * 2)) * 0.2).astype(np.float32)
    jobs = [sep.submit(mono), sep.submit(six)]
    np.testing.assert_array_equal(jobs[0].result(), sep.separate(mono))
    np.testing.assert_array_equal(jobs[1].result(), sep.separate(six))


def test_service_load_overlap3(sep):
    """Service-style load (several songs queued, overlap 3) equals one-at-a-time separation."""
    songs = [S.chunk_audio(SR * 2 + 1000 * k, seed=60 + k) for k in range(4)]
    ref = [sep.separate(m, overlap=3.0) for m in songs]
    jobs = [sep.submit(torch.from_numpy(m).pin_memory(), overlap=3.0) for m in songs]
    for r, j in zip(ref, jobs):
        np.testing.assert_array_equal(j.result(), r)


def test_queued_songs_share_forwards(sep):
    """Chunks of songs queued back to back share forwards (a song's last chunks fill a batch with the
    next song's first ones): fewer forward launches than one song at a time, identical results."""
    from turbo_roformer_b200 import _lib

    lib = _lib.load()
    songs = [S.chunk_audio(SR * 2 + 500 * k, seed=80 + k) for k in range(3)]
    counts = [sep.n_chunks(m.shape[1]) for m in songs]
    fwd_single = sum(-(-c // sep.batch) for c in counts)
    fwd_queue = -(-sum(counts) // sep.batch)
    assert fwd_queue < fwd_single  # the chunk counts are not multiples of the batch
    n0 = lib.trc_launch_count()
    ref = [sep.separate(m) for m in songs]
    n1 = lib.trc_launch_count()
    jobs = [sep.submit(m) for m in songs]
    got = [j.result() for j in jobs]
    n2 = lib.trc_launch_count()
    for r, g in zip(ref, got):
        np.testing.assert_array_equal(r, g)
    per_forward = (n1 - n0 - len(songs)) // fwd_single  # every song also makes one overlap-add launch
    assert n1 - n0 == fwd_single * per_forward + len(songs)
    assert n2 - n1 == fwd_queue * per_forward + len(songs)


def _stream_all(sep, mix, blocks, gain=1.0, overlap=2.0):
    st = sep.stream(overlap=overlap, gain=gain)
    parts, i = [], 0
    for b in blocks:
        out = st.push(mix[:, i : i + b])
        i += b
        assert out.dtype == np.float32 and out.shape[0] == 2
        assert st.samples_out == sum(p.shape[1] for p in parts) + out.shape[1]
        assert st.samples_out <= max(0, i - sep.chunk) or st.samples_out == 0
        parts.append(out)
    assert i == mix.shape[1]
    parts.append(st.close())
    return np.concatenate(parts, axis=1)


@pytest.mark.parametrize("overlap", [2.0, 3.0])
def test_stream_equals_separate(sep, overlap):
    """Blocks of every size (empty, a few samples, more than a chunk): the concatenated stream output
    equals separate() bit for bit; output lags the input by one chunk."""
    C = sep.chunk
    mix = S.chunk_audio(3 * C + 1234, seed=21)
    mix *= np.float32(0.5 / np.abs(mix).max())  # peak 0.5: separate() applies no gain
    rng = np.random.default_rng(3)
    blocks, left = [], mix.shape[1]
    while left:
        b = int(min(left, rng.choice([0, 1, 7, 441, C // 3, C, C + 5])))
        blocks.append(b)
        left -= b
    got = _stream_all(sep, mix, blocks, overlap=overlap)
    np.testing.assert_array_equal(got, sep.separate(mix, overlap=overlap))


def test_stream_with_separate_gain(sep):
    """A loud mix: with the float32 gain separate() computes (0.9 / peak), the stream matches it."""
    C = sep.chunk
    mix = S.chunk_audio(2 * C + 77, seed=22) * np.float32(2.0)
    gain = float(np.float32(0.9 / np.float64(np.abs(mix).max())))
    got = _stream_all(sep, mix, [C // 2] * 4 + [mix.shape[1] - 4 * (C // 2)], gain=gain)
    np.testing.assert_array_equal(got, sep.separate(mix))


@pytest.mark.parametrize("extra", [-300, 0, 1])
def test_stream_short_and_one_chunk(sep, extra):
    """Shorter than a chunk (the short-clip path at close), exactly one chunk, one sample more."""
    n = sep.chunk + extra
    mix = S.chunk_audio(n, seed=23) * np.float32(0.4)
    got = _stream_all(sep, mix, [n // 3, n - n // 3])
    np.testing.assert_array_equal(got, sep.separate(mix))


def test_stream_errors(sep):
    st = sep.stream()
    with pytest.raises(ValueError):
        st.push(np.full((2, 10), np.nan, np.float32))
    with pytest.raises(ValueError):
        st.push(np.zeros((3, 10), np.float32))
    with pytest.raises(ValueError):
        st.close()  # nothing pushed
    with pytest.raises(RuntimeError):
        st.push(np.zeros((2, 10), np.float32))
    with pytest.raises(ValueError):
        sep.stream(gain=0.0)
