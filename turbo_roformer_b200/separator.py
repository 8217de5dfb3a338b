"""``Separator`` with ``backend="cuda"``: the reference's public API (turbo_roformer/separator.py:57-283)
served by the B200 kernels.

Same constructor shape, same ``separate`` / ``separate_file`` / ``n_chunks`` / ``from_module`` methods,
same chunking, short-clip padding, peak normalisation to 0.9, Hamming overlap-add and
vocals = mix - instrumental. Differences: ``backend`` is ``"cuda"`` (``"auto"`` means the same), the
precision names the tensor-core operand type (``"fp16"`` default, ``"bf16"``), ``device`` picks the GPU
and ``batch`` is how many chunks share one forward call (8 by default: about 7 GB of work buffers, the
batch the throughput figures use). Weights are never downloaded by this package:
a registry name resolves to a checkpoint already present in ``model_dir``.
"""

from __future__ import annotations

import logging
import os
import threading
import time
from collections.abc import Callable
from pathlib import Path
from typing import Any

import numpy as np
import torch

from . import _lib, audio
from .backend import CudaBSRoformer
from .chunking import chunk_starts, ola_device, overlap_add_cuda, run_chunks, step_for, stream_plan
from .config import RESURRECTION, infer_config

log = logging.getLogger("turbo_roformer_b200")

SR = 44100
PEAK = 0.9
BACKENDS = ("cuda", "auto")
PRECISIONS = ("fp16", "bf16")

# registry name -> (checkpoint file name, hop, dim_t) (turbo_roformer/registry.py:71-94)
KNOWN_MODELS = {
    "resurrection": ("bs_roformer_instrumental_resurrection_unwa.ckpt", 441, 1700),
    "bs_roformer_instrumental_resurrection_unwa": ("bs_roformer_instrumental_resurrection_unwa.ckpt", 441, 1700),
    "resurrection-inst": ("bs_roformer_instrumental_resurrection_unwa.ckpt", 441, 1700),
}


def default_model_dir() -> Path:
    root = os.environ.get("TURBO_ROFORMER_HOME") or os.path.join(
        os.environ.get("XDG_CACHE_HOME", os.path.expanduser("~/.cache")), "turbo-roformer"
    )
    return Path(root) / "models"


def load_state_dict(path: str | os.PathLike) -> dict:
    """Plain state dict, or one wrapped in ``state_dict`` / ``model`` (turbo_roformer/model.py:289-297)."""
    sd = torch.load(str(path), map_location="cpu", weights_only=True)
    if isinstance(sd, dict) and isinstance(sd.get("state_dict"), dict):
        sd = sd["state_dict"]
    elif isinstance(sd, dict) and isinstance(sd.get("model"), dict):
        sd = sd["model"]
    return {k: v.float() for k, v in sd.items()}


def _hop_and_frames(cfg: dict) -> tuple[int, int]:
    """STFT hop and frames per chunk of a training config (separator.py:125-126): the hop is
    ``model.stft_hop_length`` (512 when absent); ``dim_t`` is the first one set of the ``inference`` and
    ``audio`` sections (801 when neither sets it)."""
    hop = cfg["model"].get("stft_hop_length", 512)
    sections = (cfg.get("inference") or {}, cfg.get("audio") or {})
    dim_t = next((sec["dim_t"] for sec in sections if sec.get("dim_t")), 801)
    return int(hop), int(dim_t)


class Separator:
    """Vocal/instrumental separation with a BS-RoFormer model on a B200.

    ``separate`` is serialised by an internal lock: an instance owns device work buffers, so concurrent
    calls on the same instance wait for each other.
    """

    def __init__(
        self,
        model: str = "resurrection",
        precision: str = "fp16",
        threads: int | None = None,
        model_dir: str | os.PathLike | None = None,
        *,
        backend: str = "cuda",
        config: str | os.PathLike | None = None,
        progress: bool = True,
        device: int | None = None,
        batch: int = 8,
    ):
        self._check_args(precision, backend)
        t0 = time.perf_counter()
        self.threads = threads
        if threads:
            torch.set_num_threads(int(threads))
        sd, hop, dim_t, name = self._resolve(model, model_dir, config)
        self.model_name = name
        self._configure(sd, hop, dim_t, precision, device, batch)
        self.load_s = time.perf_counter() - t0

    # ------------------------------------------------------------------ construction helpers
    @staticmethod
    def _check_args(precision: str, backend: str) -> None:
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {PRECISIONS}")
        if backend not in BACKENDS:
            raise ValueError(f"backend must be one of {BACKENDS} (the CPU backends live in the reference package)")

    @staticmethod
    def _resolve(model, model_dir, config) -> tuple[dict, int, int, str]:
        key = str(model).lower()
        if key in KNOWN_MODELS:
            fname, hop, dim_t = KNOWN_MODELS[key]
            path = Path(model_dir).expanduser() / fname if model_dir else default_model_dir() / fname
            if not path.exists():
                raise FileNotFoundError(
                    f"{path} not found: this backend does not download weights; place the checkpoint there "
                    "or pass its path with config="
                )
            return load_state_dict(path), hop, dim_t, key
        p = Path(str(model)).expanduser()
        if not p.is_file():
            raise KeyError(f"unknown model {model!r}; pass a registry name or a .ckpt path with config=")
        if config is None:
            raise ValueError("a custom checkpoint needs config=<yaml>")
        import yaml

        with open(config, encoding="utf-8") as f:
            hop, dim_t = _hop_and_frames(yaml.safe_load(f))
        return load_state_dict(p), hop, dim_t, p.name

    def _configure(self, sd, hop, dim_t, precision, device, batch) -> None:
        cfg = infer_config(sd, hop=hop, dim_t=dim_t)
        self.net = CudaBSRoformer(sd, cfg=cfg, device=device, precision=precision)
        self.cfg = cfg
        self.hop = hop
        self.chunk = hop * (dim_t - 1)
        self.backend, self.precision = "cuda", precision
        self.batch = max(1, int(batch))
        self._lock = threading.RLock()
        self._pending: list[tuple[SeparationJob, int]] = []  # queued full-length chunks: (job, chunk index)

    @classmethod
    def from_module(
        cls,
        net,
        hop: int,
        dim_t: int,
        precision: str = "fp16",
        backend: str = "cuda",
        threads: int | None = None,
        device: int | None = None,
        batch: int = 8,
    ) -> Separator:
        """Wrap an already constructed BS-RoFormer module (or its state dict) (separator.py:160-179)."""
        cls._check_args(precision, backend)
        self = cls.__new__(cls)
        self.threads = threads
        if threads:
            torch.set_num_threads(int(threads))
        sd = net if isinstance(net, dict) else net.state_dict()
        self.model_name = "custom"
        self._configure(sd, hop, dim_t, precision, device, batch)
        self.load_s = 0.0
        return self

    @classmethod
    def from_state_dict(cls, sd: dict, hop: int = RESURRECTION.stft_hop_length, dim_t: int = RESURRECTION.dim_t,
                        **kw) -> Separator:
        return cls.from_module(sd, hop, dim_t, **kw)

    # ------------------------------------------------------------------ separation
    @property
    def device(self) -> torch.device:
        return self.net.device

    def n_chunks(self, n_samples: int, overlap: float = 2.0) -> int:
        C = min(self.chunk, n_samples)
        return len(chunk_starts(n_samples, C, step_for(C, overlap)))

    def _padded_length(self, n0: int) -> int:
        """Clips shorter than one chunk are zero-padded to whole hops, at least 3 (separator.py:190-193)."""
        if n0 < self.chunk and (n0 % self.hop or n0 < 3 * self.hop):
            return max(-(-n0 // self.hop) * self.hop, 3 * self.hop)
        return n0

    def _pad_short(self, x: np.ndarray) -> np.ndarray:
        target = self._padded_length(x.shape[1])
        return np.pad(x, ((0, 0), (0, target - x.shape[1]))) if target != x.shape[1] else x

    def prepare_44k(self, x: np.ndarray) -> tuple[np.ndarray, float]:
        """Short-clip padding and peak gain (separator.py:190-197): returns (padded x * gain, gain)."""
        x = self._pad_short(x)
        peak = float(np.abs(x).max())
        gain = PEAK / peak if peak > PEAK else 1.0
        return np.ascontiguousarray(x * np.float32(gain) if gain != 1.0 else x), gain

    def separate_device(self, x: torch.Tensor, overlap: float = 2.0, progress=None, check: bool = True) -> torch.Tensor:
        """(2, n) float32 already on the model's GPU (padded and gain-applied) -> (2, n) on the GPU.

        With ``check=False`` the call only queues work (no host synchronisation); ``self.net.check()``
        later synchronises and raises any device-side error."""
        return overlap_add_cuda(self.net, x, self.chunk, overlap, batch=self.batch, progress=progress, check=check)

    @staticmethod
    def _pinned(x) -> torch.Tensor:
        """A pinned float32 CPU tensor holding x (numpy or CPU tensor); a pinned tensor is used as is."""
        if isinstance(x, torch.Tensor) and x.is_pinned() and x.dtype == torch.float32 and x.is_contiguous():
            return x
        a = np.ascontiguousarray(x.numpy() if isinstance(x, torch.Tensor) else x, dtype=np.float32)
        src = torch.empty(a.shape, dtype=torch.float32, pin_memory=True)
        src.numpy()[...] = a
        return src

    @torch.inference_mode()
    def _submit_44k(self, x, overlap: float, progress, out: torch.Tensor | None) -> "SeparationJob":
        """separator.py:186-200 queued on the GPU without a host synchronisation.

        The samples are copied to the GPU once (from pinned memory: the caller's, or a pinned staging
        copy of a numpy mix). ``x`` is (2, n) float32: numpy or a CPU tensor."""
        n0 = x.shape[1]
        if not (isinstance(x, torch.Tensor) and x.is_pinned() and n0 >= self.chunk):
            x = self._pad_short(x.numpy() if isinstance(x, torch.Tensor) else x)
        src = self._pinned(x)
        return self._submit_device(src.to(self.device, non_blocking=True), n0, overlap, progress, out, src)

    @torch.inference_mode()
    def _submit_resampled(self, x: np.ndarray, sr: int, overlap: float, progress,
                          out: torch.Tensor | None = None) -> "SeparationJob":
        """Any channel count and sample rate: the channel fold and both rate conversions on the GPU
        (``resample.remix_device`` / ``resample_device``), the 44.1 kHz part as ``_submit_44k``.
        The reference does these on the host (separator.py:214-230, audio.py:35-82)."""
        from .resample import remix_device, resample_device

        n = x.shape[1]
        src = self._pinned(x)
        xd = remix_device(src.to(self.device, non_blocking=True))
        if sr != SR:
            xd = resample_device(xd, sr, SR, length=max(1, round(n * SR / sr)))
        n0 = xd.shape[1]
        xd = torch.nn.functional.pad(xd, (0, self._padded_length(n0) - n0)).contiguous()
        post = (lambda inst: resample_device(inst.contiguous(), SR, sr, length=n)) if sr != SR else None
        if out is None:
            out = torch.empty((2, n), dtype=torch.float32, pin_memory=True)
        return self._submit_device(xd, n0, overlap, progress, out, src, post)

    def _submit_device(self, xd: torch.Tensor, n0: int, overlap: float, progress, out: torch.Tensor | None,
                       src: torch.Tensor, post=None) -> "SeparationJob":
        """The part of separator.py:186-200 after the upload: ``xd`` (2, n) on the GPU, already padded;
        the first n0 samples are the song. The peak gain PEAK / max|x| (rounded from double to float32,
        as the host code computes it) multiplies the mix and divides the instrumental on the device, the
        NaN/inf scan is max|x| being finite (NaN propagates through the maximum), and one asynchronous
        copy returns the instrumental (through ``post`` if given) into pinned host memory."""
        n_res = out.shape[1] if (post is not None and out is not None) else n0
        if out is None:
            out = torch.empty((2, n_res), dtype=torch.float32, pin_memory=True)
        elif out.shape != (2, n_res) or out.dtype != torch.float32 or not out.is_pinned() or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous pinned float32 CPU tensor of shape (2, {n_res})")
        flags = torch.zeros(2, dtype=torch.int32, pin_memory=True)  # [device error word, non-finite input]
        peak = xd.abs().amax()
        gain = torch.where(peak > PEAK, (PEAK / peak.double()).float(), torch.ones((), device=xd.device))
        xd.mul_(gain)
        n = xd.shape[1]
        C = min(self.chunk, n)
        starts = chunk_starts(n, C, step_for(C, overlap))
        job = SeparationJob(self, out, flags)
        job._song = _Song(xd, starts, C, n0, gain, peak, torch.empty(len(starts), 2, self.net.output_length(C),
                                                                    device=xd.device, dtype=torch.float32), src)
        job._song.post = post
        if C != self.chunk or progress is not None:
            # a short clip (its own chunk length) or a caller that follows the chunks: its own forwards
            run_chunks(self.net, xd, starts, C, self.batch, job._song.outs, progress, check=False)
            job._song.left = 0
            self._finish(job)
        else:
            self._pending.extend((job, i) for i in range(len(starts)))
            self._run_pending(full_only=True)
        return job

    def _run_pending(self, full_only: bool) -> None:
        """Forward the queued chunks ``batch`` at a time, whichever songs they come from (a song's last
        chunks share a forward with the next song's first ones); the outputs go to each song's chunk
        buffer and a song whose chunks are all done is overlap-added and copied back. With
        ``full_only`` a partial batch stays queued for the next song. Forward outputs do not depend on
        which chunks share a batch, so the result equals one song at a time bit for bit."""
        while len(self._pending) >= self.batch or (not full_only and self._pending):
            sel = self._pending[: self.batch]
            del self._pending[: self.batch]
            frames = torch.stack([j._song.xd[:, j._song.starts[i] : j._song.starts[i] + j._song.C] for j, i in sel])
            y = self.net.forward_device(frames, check=False)
            for k, (j, i) in enumerate(sel):
                j._song.outs[i].copy_(y[k])
                j._song.left -= 1
                if j._song.left == 0:
                    self._finish(j)

    def _finish(self, job: "SeparationJob") -> None:
        """Overlap-add, undo the gain, copy the instrumental back and read the error words (queued)."""
        g = job._song
        inst = ola_device(g.outs, g.starts, g.C, g.n)
        inst.div_(g.gain)
        res = inst[:, : g.n0] if g.post is None else g.post(inst[:, : g.n0])
        job._out.copy_(res, non_blocking=True)
        job._flags[1:].copy_((~torch.isfinite(g.peak)).to(torch.int32).reshape(1), non_blocking=True)
        self.net.error_async(job._flags[:1])
        job._done = torch.cuda.Event()
        job._done.record(torch.cuda.current_stream(self.device))
        job._keep = (g, inst, res)
        job._song = None

    def flush(self) -> None:
        """Run the chunks still waiting for a full batch (``job.result()`` does this when it needs to)."""
        with self._lock, torch.inference_mode():
            self._run_pending(full_only=False)

    def _separate_44k(self, x: np.ndarray, overlap: float, progress) -> np.ndarray:
        return self._submit_44k(x, overlap, progress, None).result()

    def submit(self, mix, overlap: float = 2.0, out: torch.Tensor | None = None) -> "SeparationJob":
        """Queue one song on the GPU and return at once; ``job.result()`` waits for it.

        Same input contract and result as ``separate`` for 44.1 kHz input (no resampling here; mono and
        surround layouts are folded to stereo on the GPU). Several
        songs may be queued back to back: the host never synchronises between them, so the GPU stays busy
        while the host prepares the next song. A mix in pinned memory (a pinned CPU tensor) is copied by
        DMA straight from the caller's buffer; ``out`` may supply a pinned (2, n) float32 result buffer.
        A service streaming many songs through one Separator is the intended user (no reference
        counterpart: the reference separates one song per call)."""
        if not overlap >= 1.0:
            raise ValueError("overlap must be >= 1")
        if isinstance(mix, torch.Tensor):
            if mix.device.type != "cpu" or mix.dtype != torch.float32 or mix.ndim != 2 or mix.shape[0] != 2:
                raise ValueError("a tensor mix must be a (2, n) float32 CPU tensor")
            if mix.shape[1] == 0:
                raise ValueError("empty input")
            x = mix.contiguous()
        else:
            x = audio.as_channels_first(mix, finite=False)
            if x.shape[0] != 2:
                with self._lock:
                    return self._submit_resampled(x, SR, float(overlap), None, out)
        with self._lock:
            return self._submit_44k(x, float(overlap), None, out)

    def stream(self, overlap: float = 2.0, gain: float = 1.0) -> "SeparationStream":
        """Separate a 44.1 kHz stereo stream as it arrives: ``push`` blocks, ``close`` at the end.

        The streaming API of the reference's roadmap (README.md:139). The chunk schedule, overlap-add and
        forward are ``separate``'s, so the blocks the stream returns, concatenated, equal
        ``separate(whole_mix)`` bit for bit whenever ``gain`` is the gain ``separate`` applies (1.0 for a
        mix whose peak is at most 0.9; else the float32 value of 0.9 / peak). A stream cannot see the
        peak ahead of time, so the caller chooses the gain. Output lags the input by one chunk."""
        if not overlap >= 1.0:
            raise ValueError("overlap must be >= 1")
        if not (np.isfinite(gain) and gain > 0):
            raise ValueError("gain must be a positive finite number")
        return SeparationStream(self, float(overlap), float(gain))

    def separate(
        self,
        mix,
        sr: int = SR,
        overlap: float = 2.0,
        progress: Callable[[int, int], None] | None = None,
    ) -> np.ndarray:
        """Instrumental as float32 (2, samples) at ``sr``; vocals = ``to_stereo(mix) - inst`` (separator.py:203-232)."""
        if not overlap >= 1.0:
            raise ValueError("overlap must be >= 1")
        if int(sr) <= 0:
            raise ValueError("sr must be positive")
        sr = int(sr)
        x = audio.as_channels_first(mix, finite=False)
        with self._lock:
            if self.threads:
                torch.set_num_threads(int(self.threads))
            if sr == SR and x.shape[0] == 2:
                return self._separate_44k(x, float(overlap), progress)
            # fold and rate conversion on the GPU around the 44.1 kHz model
            return self._submit_resampled(x, sr, float(overlap), progress).result()

    def separate_file(
        self,
        in_path: str | os.PathLike,
        out_dir: str | os.PathLike,
        formats: tuple[str, ...] | list[str] = ("wav",),
        overlap: float = 2.0,
        progress: Callable[[int, int], None] | None = None,
    ) -> dict[str, Any]:
        """Decode ``in_path``, separate it and write ``<stem>_instrumental.<fmt>`` and ``<stem>_vocals.<fmt>``
        into ``out_dir`` for every format (separator.py:234-283).

        Returns the first format's two paths (``instrumental``, ``vocals``), every path under ``files``
        (keyed ``"<name>.<fmt>"``), the phase times ``read_s`` / ``separate_s`` / ``write_s`` / ``wall_s``,
        ``rtf`` = wall_s / duration_s, ``sample_rate``, ``n_chunks`` (at 44.1 kHz), ``backend`` and
        ``precision``. Unknown or missing formats raise ``ValueError`` before the file is read."""
        formats = tuple(formats)
        if not formats:
            raise ValueError("at least one output format is needed")
        for fmt in formats:
            if fmt not in audio.output_formats():
                raise ValueError(f"unsupported output format {fmt!r}")
        clock = [time.perf_counter()]
        decoded, sr = audio.load(in_path)
        clock.append(time.perf_counter())
        mix = audio.to_stereo(audio.as_channels_first(decoded))
        inst = self.separate(mix, sr=sr, overlap=overlap, progress=progress)
        stems = {"instrumental": inst, "vocals": mix - inst}
        clock.append(time.perf_counter())
        files = _write_stems(Path(out_dir), Path(in_path).stem, stems, sr, formats)
        clock.append(time.perf_counter())
        read_s, separate_s, write_s = (b - a for a, b in zip(clock, clock[1:]))
        wall_s = clock[-1] - clock[0]
        duration_s = mix.shape[1] / sr
        first = formats[0]
        return {
            "instrumental": files[f"instrumental.{first}"],
            "vocals": files[f"vocals.{first}"],
            "files": files,
            "duration_s": duration_s,
            "sample_rate": sr,
            "n_chunks": self.n_chunks(round(mix.shape[1] * SR / sr), overlap),  # the 44.1 kHz length run
            "read_s": read_s,
            "separate_s": separate_s,
            "write_s": write_s,
            "wall_s": wall_s,
            "rtf": wall_s / duration_s,
            "backend": self.backend,
            "precision": self.precision,
        }


def _write_stems(out: Path, stem: str, stems: dict[str, np.ndarray], sr: int, formats: tuple[str, ...]) -> dict[str, str]:
    """Encode each stem in each format as ``out/<stem>_<name>.<fmt>``; returns ``{"<name>.<fmt>": path}``."""
    out.mkdir(parents=True, exist_ok=True)
    files: dict[str, str] = {}
    for fmt in formats:
        for name, data in stems.items():
            path = out / f"{stem}_{name}.{fmt}"
            audio.write(path, data, sr, fmt)
            files[f"{name}.{fmt}"] = str(path)
    return files


class _Song:
    """A queued song's device state until its overlap-add is queued."""

    def __init__(self, xd, starts, C, n0, gain, peak, outs, src):
        self.xd, self.starts, self.C, self.n0, self.gain, self.peak, self.outs, self.src = (
            xd, starts, C, n0, gain, peak, outs, src)
        self.n = xd.shape[1]
        self.left = len(starts)
        self.post = None  # device transform of the instrumental before the copy back (rate conversion)


class SeparationJob:
    """A song queued by ``Separator.submit``. ``result()`` waits for it and returns the instrumental.

    Chunks of songs queued back to back share forwards, so a song's last chunks may wait for the next
    song's (or for ``result()`` / ``Separator.flush()``) to fill a batch."""

    def __init__(self, sep: Separator, out: torch.Tensor, flags: torch.Tensor):
        self._sep, self._out, self._flags = sep, out, flags
        self._done: torch.cuda.Event | None = None
        self._song: _Song | None = None
        self._keep = None

    def done(self) -> bool:
        """True once the GPU has finished the song (non-blocking)."""
        return self._done is not None and self._done.query()

    def result(self) -> np.ndarray:
        """float32 (2, n) instrumental (a view of the pinned result buffer); raises ValueError on NaN/inf
        input and TRCError if a kernel reported a device-side error (a forward shared with another song
        reports to the first of the songs that finish after it)."""
        if self._done is None:
            self._sep.flush()
        self._done.synchronize()
        self._keep = None
        err, nonfinite = (int(v) for v in self._flags.tolist())
        if err:
            raise _lib.TRCError(_lib.TRC_E_DEVICE, f"device error {err} reported by a kernel (bounded wait expired)")
        if nonfinite:
            raise ValueError("input contains NaN or inf samples")
        return self._out.numpy()


class SeparationStream:
    """Incremental separation (``Separator.stream``): ``push(block)`` returns the instrumental samples that
    became final, ``close()`` the rest.

    Regular chunks run as soon as all of their samples and one more have arrived (their start s has
    s + chunk < samples so far, so they belong to the final schedule); a sample is final once it lies
    before the last chunk length of the input, which the tail chunk (aligned to the end) cannot reach.
    Each returned segment is the device overlap-add of every chunk that covers it, in start order, so its
    values are those of the whole-song overlap-add. Only the samples later chunks still read and the
    outputs of chunks that reach past the returned samples stay on the GPU."""

    def __init__(self, sep: Separator, overlap: float, gain: float):
        self._sep = sep
        self._C = sep.chunk
        self._overlap = overlap
        self._step = step_for(self._C, overlap)
        self._gain = torch.tensor(gain, dtype=torch.float32, device=sep.device)
        self._x = torch.empty(2, 0, device=sep.device, dtype=torch.float32)  # samples [_base, _n), gain applied
        self._base = 0
        self._n = 0
        self._next = 0                     # next regular chunk start
        self._starts: list[int] = []       # chunks whose outputs are still needed, in start order
        self._outs: list[torch.Tensor] = []
        self._emitted = 0
        self._closed = False

    @property
    def samples_in(self) -> int:
        return self._n

    @property
    def samples_out(self) -> int:
        return self._emitted

    def _block(self, block) -> torch.Tensor:
        a = block.numpy() if isinstance(block, torch.Tensor) else np.asarray(block)
        if a.dtype.kind != "f":
            raise ValueError(f"expected floating point samples, got dtype {a.dtype}")
        if a.ndim == 1:
            a = np.stack([a, a])
        if a.ndim != 2 or a.shape[0] != 2:
            raise ValueError(f"expected a (2, samples) or (samples,) block, got shape {a.shape}")
        audio.check_finite(a)
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))

    def push(self, block) -> np.ndarray:
        """Append a (2, k) float32 block (or mono (k,)); returns the (2, m) instrumental samples now final."""
        if self._closed:
            raise RuntimeError("stream is closed")
        xb = self._block(block)
        if xb.shape[1] == 0:
            return np.zeros((2, 0), np.float32)
        with self._sep._lock, torch.inference_mode():
            xd = xb.to(self._sep.device).mul_(self._gain)
            self._x = torch.cat([self._x, xd], dim=1)
            self._n += xd.shape[1]
            starts, end = stream_plan(self._n, self._next, self._C, self._step, final=False)
            if starts:
                self._next = starts[-1] + self._step
            return self._advance(starts, end)

    def close(self) -> np.ndarray:
        """End of input: run the remaining chunks and return the rest of the instrumental."""
        if self._closed:
            raise RuntimeError("stream is closed")
        self._closed = True
        if self._n == 0:
            raise ValueError("empty input")
        with self._sep._lock, torch.inference_mode():
            if self._n < self._C:  # a clip shorter than one chunk: the separator's short-clip path
                sep = self._sep
                xd = torch.nn.functional.pad(self._x, (0, sep._padded_length(self._n) - self._n))
                inst = overlap_add_cuda(sep.net, xd, sep.chunk, self._overlap, batch=sep.batch)
                inst.div_(self._gain)
                self._emitted = self._n
                return inst[:, : self._n].cpu().numpy()
            starts, end = stream_plan(self._n, self._next, self._C, self._step, final=True)
            return self._advance(starts, end)

    def _advance(self, starts: list[int], end: int) -> np.ndarray:
        sep, C = self._sep, self._C
        for b0 in range(0, len(starts), sep.batch):
            sel = starts[b0 : b0 + sep.batch]
            frames = torch.stack([self._x[:, s - self._base : s - self._base + C] for s in sel])
            y = sep.net.forward_device(frames, check=False)
            self._starts += sel
            self._outs += list(y)
        if end <= self._emitted:
            sep.net.check()
            return np.zeros((2, 0), np.float32)
        # the chunks that cover [_emitted, end): all kept chunks from the first one reaching past _emitted
        L = sep.net.output_length(C)
        first = next(i for i, s in enumerate(self._starts) if s + L > self._emitted)
        last = max(i for i, s in enumerate(self._starts) if s < end)
        s0 = self._starts[first]
        rel = [s - s0 for s in self._starts[first : last + 1]]
        ola = ola_device(torch.stack(self._outs[first : last + 1]), rel, C, rel[-1] + C)
        seg = ola[:, self._emitted - s0 : end - s0].div_(self._gain).cpu().numpy()
        sep.net.check()
        self._emitted = end
        # drop what later segments no longer read: chunk outputs that end at or before `end`, and the
        # input before the earliest start a later chunk can have (the next regular start or the tail's)
        keep = [i for i, s in enumerate(self._starts) if s + L > end]
        self._starts = [self._starts[i] for i in keep]
        self._outs = [self._outs[i] for i in keep]
        cut = min(self._next, max(0, self._n - C)) - self._base
        if cut > 0:
            self._x = self._x[:, cut:].contiguous()
            self._base += cut
        return seg
