"""Host-side Separator logic that needs no GPU: input validation, channel handling, padding and peak gain,
and the loud failure when the CUDA backend is unavailable."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import chunking_oracle as O
from turbo_roformer_b200 import audio
from turbo_roformer_b200.separator import Separator


@pytest.mark.parametrize(
    "bad",
    [
        np.array([[0.0, np.nan, 0.0]] * 2, np.float32),
        np.array([[0.0, np.inf, 0.0]] * 2, np.float32),
        np.zeros((2, 0), np.float32),
        np.zeros((2, 10), np.int16),
        np.zeros((1000, 2), np.float32),
        np.zeros((2, 2, 10), np.float32),
    ],
)
def test_invalid_input_raises(bad):
    with pytest.raises(ValueError):
        audio.as_channels_first(bad)


def _fold_by_rule(x):
    """The separator's surround fold written out channel by channel (turbo_roformer/audio.py:35-59):
    centre to both sides at -3 dB, LFE of >= 6 channels dropped, the rest alternately left/right at
    -3 dB, each side divided by its summed gains."""
    g = 0.7071
    sides = [[(0, 1.0)], [(1, 1.0)]]
    if x.shape[0] >= 3:
        sides[0].append((2, g))
        sides[1].append((2, g))
    for k, ch in enumerate(range(4 if x.shape[0] >= 6 else 3, x.shape[0])):
        sides[k % 2].append((ch, g))
    out = [sum(w * x[ch].astype(np.float64) for ch, w in s) / sum(w for _, w in s) for s in sides]
    return np.stack(out).astype(np.float32)


@pytest.mark.parametrize("channels", [3, 4, 5, 6, 7, 8, 16])
def test_surround_fold_matches_the_channel_rule(channels):
    rng = np.random.default_rng(channels)
    x = rng.standard_normal((channels, 1000)).astype(np.float32)
    np.testing.assert_allclose(audio.to_stereo(x), _fold_by_rule(x), rtol=1e-6, atol=1e-7)
    if channels >= 6:  # the LFE never reaches the output
        lfe_only = np.zeros_like(x)
        lfe_only[3] = x[3]
        assert not audio.to_stereo(lfe_only).any()


def test_downmix_keeps_centre():
    rng = np.random.default_rng(2)
    six = rng.standard_normal((6, 1000)).astype(np.float32)
    centre_only = np.zeros_like(six)
    centre_only[2] = six[2]
    dm = audio.downmix_stereo(centre_only)
    assert np.abs(dm).max() > 0.2 * np.abs(six[2]).max()
    np.testing.assert_allclose(dm[0], dm[1])
    assert audio.to_stereo(six).shape == (2, 1000)
    mono = six[:1]
    np.testing.assert_array_equal(audio.to_stereo(mono), np.repeat(mono, 2, axis=0))
    stereo = six[:2]
    np.testing.assert_array_equal(audio.to_stereo(stereo), stereo)


def test_resample_length_rule_without_rate_change():
    x = np.arange(20, dtype=np.float32).reshape(2, 10)
    np.testing.assert_array_equal(audio.resample(x, 44100, 44100, length=7), x[:, :7])
    padded = audio.resample(x, 44100, 44100, length=12)
    np.testing.assert_array_equal(padded[:, :10], x)
    assert not padded[:, 10:].any()


def _bare(chunk=16256, hop=128):
    s = Separator.__new__(Separator)
    s.chunk, s.hop = chunk, hop
    return s


@pytest.mark.parametrize("n", [1, 2, 127, 128, 383, 385, 16255, 16256, 16257])
def test_short_clip_padding_and_gain_match_reference_rules(n):
    rng = np.random.default_rng(n)
    x = (3.0 * rng.standard_normal((2, n))).astype(np.float32)
    s = _bare()
    xp, gain = s.prepare_44k(x)
    captured = {}

    def run(c):
        captured.setdefault("first", c.clone())
        return c

    O.separate_44k(x, s.chunk, s.hop, 2.0, run)  # the oracle pads/gains identically before its first chunk
    assert xp.shape[1] >= n
    first = captured["first"][0].numpy()
    np.testing.assert_array_equal(xp[:, : first.shape[1]], first)
    if np.abs(x).max() > 0.9:
        assert gain == pytest.approx(0.9 / np.abs(x).max())


def test_backend_and_precision_validation():
    with pytest.raises(ValueError):
        Separator._check_args("fp32", "cuda")
    with pytest.raises(ValueError):
        Separator._check_args("fp16", "torch")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure mode")
def test_cuda_backend_fails_loudly_without_gpu(tiny_sd):
    from turbo_roformer_b200._lib import KernelUnavailable

    with pytest.raises(KernelUnavailable):
        Separator.from_module(tiny_sd, 128, 128)


class _FakeNet:
    """A batch-invariant stand-in for the CUDA model on the CPU: y = tanh(3 x) over whole hops."""

    hop = 7

    def output_length(self, n):
        return self.hop * (n // self.hop)

    def forward_device(self, frames, out=None, check=True):
        y = torch.tanh(frames[..., : self.output_length(frames.shape[-1])] * 3.0)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def check(self):
        pass


def _fake_separator(monkeypatch, chunk, batch):
    import threading

    monkeypatch.setattr(Separator, "device", property(lambda self: torch.device("cpu")))
    sep = Separator.__new__(Separator)
    sep.net, sep.chunk, sep.hop, sep.batch = _FakeNet(), chunk, _FakeNet.hop, batch
    sep._lock = threading.RLock()
    sep._pending = []
    return sep


@pytest.mark.parametrize("overlap,batch", [(2.0, 1), (3.0, 3), (1.5, 2)])
def test_stream_logic_matches_whole_song_overlap_add(monkeypatch, overlap, batch):
    """Separator.stream on a CPU stand-in model (the device overlap-add replaced by the oracle's loop):
    the concatenated blocks equal the whole-song overlap-add of the same model bit for bit."""
    from turbo_roformer_b200 import separator as SP

    monkeypatch.setattr(SP, "ola_device", lambda ys, starts, C, n: O.ola_from_outputs(list(ys), starts, n, C))
    monkeypatch.setattr(SP, "overlap_add_cuda", lambda net, x, chunk, ov, batch: O.overlap_add(x, chunk, ov, net.forward_device))
    C = 7 * 40
    sep = _fake_separator(monkeypatch, C, batch)
    rng = np.random.default_rng(5)
    for n in (5, 30, C - 3, C, C + 1, 3 * C + 17, 5 * C):
        mix = rng.standard_normal((2, n)).astype(np.float32)
        mix *= np.float32(0.5 / np.abs(mix).max())
        ref = O.separate_44k(mix, C, _FakeNet.hop, overlap, sep.net.forward_device)
        st = sep.stream(overlap=overlap)
        parts, i = [], 0
        while i < n:
            b = int(rng.choice([0, 1, 5, 33, C // 2, C + 3]))
            parts.append(st.push(mix[:, i : i + b]))
            i += b
            assert st.samples_out == max(0, min(i, n) - C)
        parts.append(st.close())
        np.testing.assert_array_equal(np.concatenate(parts, axis=1), ref)


class _FakeSoundfile:
    """In-memory stand-in for the optional 'soundfile' package: read returns a stored (samples, channels)
    array, write records what would have been encoded."""

    def __init__(self, frames, sr):
        self.frames, self.sr, self.written = frames, sr, {}

    def read(self, path, dtype="float32", always_2d=True):
        assert dtype == "float32" and always_2d
        return self.frames.copy(), self.sr

    def write(self, path, data, sr, subtype=None, format=None):
        self.written[path] = (np.array(data), sr, subtype, format)


@pytest.mark.parametrize("channels,sr", [(2, 44100), (1, 48000), (6, 44100)])
def test_separate_file_writes_stems_and_reports(monkeypatch, tmp_path, channels, sr):
    """separate_file (separator.py:234-283) on a stand-in decoder and model: the stems are the folded mix's
    instrumental and mix - instrumental, written per format as <stem>_<name>.<fmt> with the reference's
    encodings, and the result carries the reference's keys."""
    import sys

    rng = np.random.default_rng(channels)
    frames = (0.3 * rng.standard_normal((5000, channels))).astype(np.float32)
    sf = _FakeSoundfile(frames, sr)
    monkeypatch.setitem(sys.modules, "soundfile", sf)
    seen = {}

    def fake_separate(self, mix, sr=44100, overlap=2.0, progress=None):
        seen.update(mix=mix.copy(), sr=sr, overlap=overlap)
        return (0.25 * mix).astype(np.float32)

    monkeypatch.setattr(Separator, "separate", fake_separate)
    sep = _bare(chunk=1000, hop=10)
    sep.backend, sep.precision = "cuda", "fp16"
    res = sep.separate_file(tmp_path / "song.flac", tmp_path / "out", formats=("wav", "flac"), overlap=3.0)

    mix = audio.to_stereo(frames.T)
    np.testing.assert_array_equal(seen["mix"], mix)
    assert seen["sr"] == sr and seen["overlap"] == 3.0
    inst = (0.25 * mix).astype(np.float32)
    expect = {"instrumental": inst, "vocals": mix - inst}
    assert set(res["files"]) == {"instrumental.wav", "vocals.wav", "instrumental.flac", "vocals.flac"}
    for key, path in res["files"].items():
        name, fmt = key.split(".")
        assert path == str(tmp_path / "out" / f"song_{name}.{fmt}")
        data, w_sr, subtype, container = sf.written[path]
        np.testing.assert_array_equal(data, expect[name].T)
        assert (w_sr, subtype, container) == (sr, audio.FORMATS[fmt], fmt.upper())
    assert res["instrumental"] == res["files"]["instrumental.wav"] and res["vocals"] == res["files"]["vocals.wav"]
    assert (tmp_path / "out").is_dir()
    assert res["sample_rate"] == sr and res["duration_s"] == pytest.approx(5000 / sr)
    assert res["n_chunks"] == sep.n_chunks(round(5000 * 44100 / sr), 3.0)
    assert res["backend"] == "cuda" and res["precision"] == "fp16"
    for k in ("read_s", "separate_s", "write_s"):
        assert res[k] >= 0.0
    assert res["wall_s"] == pytest.approx(res["read_s"] + res["separate_s"] + res["write_s"])
    assert res["rtf"] == pytest.approx(res["wall_s"] / res["duration_s"])


@pytest.mark.parametrize("formats", [("mp3",), ("wav", "ogg"), ()])
def test_separate_file_rejects_formats_before_reading(monkeypatch, tmp_path, formats):
    import sys

    sf = _FakeSoundfile(np.zeros((10, 2), np.float32), 44100)
    monkeypatch.setitem(sys.modules, "soundfile", sf)
    monkeypatch.setattr(sf, "read", lambda *a, **k: pytest.fail("read before the formats were checked"))
    with pytest.raises(ValueError):
        _bare().separate_file(tmp_path / "x.wav", tmp_path, formats=formats)
    assert not sf.written


def test_training_config_hop_and_frames_defaults():
    """The reference's config defaults (separator.py:125-126): hop 512, dim_t from inference, then audio,
    then 801; a zero or missing dim_t falls through to the next section."""
    from turbo_roformer_b200.separator import _hop_and_frames

    assert _hop_and_frames({"model": {}}) == (512, 801)
    assert _hop_and_frames({"model": {"stft_hop_length": 441}, "audio": {"dim_t": 1101}}) == (441, 1101)
    assert _hop_and_frames({"model": {}, "inference": {"dim_t": 1700}, "audio": {"dim_t": 3}}) == (512, 1700)
    assert _hop_and_frames({"model": {}, "inference": {"dim_t": 0}, "audio": {"dim_t": 5}}) == (512, 5)
    assert _hop_and_frames({"model": {}, "inference": None}) == (512, 801)


def test_model_resolution_errors(tmp_path):
    """No downloads: a registry name without its checkpoint in model_dir, an unknown name, and a custom
    checkpoint without its config each fail before any device work."""
    with pytest.raises(FileNotFoundError):
        Separator._resolve("resurrection", tmp_path, None)
    with pytest.raises(KeyError):
        Separator._resolve("no-such-model", tmp_path, None)
    ckpt = tmp_path / "custom.ckpt"
    ckpt.write_bytes(b"")
    with pytest.raises(ValueError):
        Separator._resolve(str(ckpt), None, None)
