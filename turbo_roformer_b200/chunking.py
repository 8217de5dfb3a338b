"""Chunk schedule and Hamming overlap-add (the contract of turbo_roformer/chunking.py:11-61).

``chunk_starts`` / ``step_for`` / ``hamming`` follow the reference's schedule exactly (regular steps of
floor(chunk / overlap), tail chunk aligned to the end; symmetric Hamming window). ``overlap_add`` keeps the
reference's signature for any ``run`` callable on CUDA tensors; ``overlap_add_cuda`` is the device path used
by the CUDA backend: chunks are batched through one model call per batch. Both sum in libtrcuda's
overlap-add kernel, which accumulates in start order with separately rounded multiplies and adds, so
the result is bit-identical to the reference's loop for identical chunk outputs.
"""

from __future__ import annotations

import ctypes
from collections.abc import Callable

import numpy as np
import torch

from . import _lib


def chunk_starts(n: int, chunk: int, step: int) -> list[int]:
    """Offsets 0, step, 2 step, ... while a full chunk fits; then one chunk ending at n (chunking.py:11-21)."""
    if n <= 0 or chunk <= 0 or step <= 0:
        raise ValueError("n, chunk and step must be positive")
    out: list[int] = []
    off = 0
    while off < n:
        if off + chunk >= n:
            last = max(n - chunk, 0)
            if not out or out[-1] != last:
                out.append(last)
            break
        out.append(off)
        off += step
    return out


def step_for(chunk: int, overlap: float) -> int:
    """floor(chunk / overlap) clamped to [1, chunk] (chunking.py:31-33)."""
    return max(1, min(chunk, int(chunk / overlap)))


def hamming(n: int) -> np.ndarray:
    """Symmetric Hamming window 0.54 - 0.46 cos(2 pi k / (n - 1)), float32 (chunking.py:24-28)."""
    if n == 1:
        return np.ones(1, np.float32)
    k = np.arange(n, dtype=np.float64)
    return (0.54 - 0.46 * np.cos(2.0 * np.pi * k / (n - 1))).astype(np.float32)


def stream_plan(n: int, next_start: int, chunk: int, step: int, final: bool) -> tuple[list[int], int]:
    """One step of streaming the schedule of ``chunk_starts`` while the length is still growing.

    ``n`` samples have arrived, the regular chunks before ``next_start`` have run. Returns the starts to
    run now and the end of the samples that are final after them. A regular start s is certain once
    s + chunk < n (the total only grows); the tail chunk ends at the total length, so it starts at or after
    n - chunk, and every sample before n - chunk has all of its chunks among the regular ones. With
    ``final`` the length is n: the rest of ``chunk_starts(n, chunk, step)`` runs and everything is final;
    the tail chunk may start before ``next_start`` (it starts after every regular chunk that ran, since
    those end before n). (Requires n >= chunk when ``final``: a shorter clip takes the separator's
    short-clip path.)"""
    if final:
        return [s for s in chunk_starts(n, chunk, step) if not (s < next_start and s % step == 0)], n
    starts = []
    s = next_start
    while s + chunk < n:
        starts.append(s)
        s += step
    return starts, max(0, n - chunk)


def overlap_add(
    x: torch.Tensor,
    chunk: int,
    overlap: float,
    run: Callable[[torch.Tensor], torch.Tensor],
    progress: Callable[[int, int], None] | None = None,
) -> torch.Tensor:
    """x (2, n) -> (2, n): the reference's helper (chunking.py:36-61) with the weighted sum on the GPU.

    ``run`` maps (1, 2, C) -> (1, 2, L); the first min(C, L) samples are kept, L the same for every chunk.
    A CUDA model (``CudaBSRoformer``: it has ``forward_device``) takes the batched device path and x may
    then be on the host (the result comes back to x's device). Any other ``run`` is called once per chunk,
    in start order, on slices of x, which must already be a CUDA tensor; its outputs are summed by
    libtrcuda's overlap-add kernel (start order, separately rounded multiply and add: bit-identical to
    the reference's loop for the same chunk outputs). There is no host-side overlap-add."""
    if hasattr(run, "forward_device"):
        xd = x.to(device=run.device, dtype=torch.float32).contiguous()
        return overlap_add_cuda(run, xd, chunk, overlap, progress=progress).to(x.device)
    if not x.is_cuda:
        raise ValueError("overlap_add sums on the GPU: pass x as a CUDA tensor, or a CudaBSRoformer as run")
    n = x.shape[1]
    C = min(chunk, n)
    starts = chunk_starts(n, C, step_for(C, overlap))
    ys = []
    for i, s in enumerate(starts):
        y = run(x[:, s : s + C].unsqueeze(0).contiguous())[0]
        ys.append(y[:, : min(C, y.shape[-1])])
        if progress is not None:
            progress(i + 1, len(starts))
    if len({tuple(y.shape) for y in ys}) != 1 or ys[0].shape[0] != 2:
        raise ValueError("run must return (1, 2, L) with the same L for every chunk")
    chunks = torch.stack([y.to(device=x.device, dtype=torch.float32) for y in ys])
    return ola_device(chunks, starts, C, n)


def ola_device(chunks: torch.Tensor, starts: list[int], chunk: int, n: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Weighted overlap-add of device chunk outputs (n_chunks, 2, L) at ``starts`` -> (2, n) on the same device."""
    if chunks.ndim != 3 or chunks.shape[1] != 2 or not chunks.is_cuda or chunks.dtype != torch.float32:
        raise ValueError("chunks must be a float32 CUDA tensor (n_chunks, 2, L)")
    chunks = chunks.contiguous()
    lib = _lib.load()
    if out is None:
        out = torch.empty(2, n, device=chunks.device, dtype=torch.float32)
    st = (ctypes.c_int64 * len(starts))(*starts)
    with torch.cuda.device(chunks.device):
        _lib.check(
            lib.trc_ola(
                ctypes.c_void_p(chunks.data_ptr()),
                chunks.shape[2],
                st,
                len(starts),
                chunk,
                n,
                ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(torch.cuda.current_stream(chunks.device).cuda_stream),
            )
        )
    return out


def run_chunks(model, x: torch.Tensor, starts: list[int], C: int, batch: int, out: torch.Tensor,
               progress: Callable[[int, int], None] | None = None, total: int | None = None, done0: int = 0,
               check: bool = True) -> None:
    """Forward the chunks x[:, s:s+C] for s in starts through ``model`` in batches, into out[i].

    ``check=False`` leaves the device-error check (a stream synchronisation) to the caller, so a caller
    that queues several songs keeps the GPU fed while the host runs ahead."""
    total = total if total is not None else len(starts)
    for b0 in range(0, len(starts), batch):
        sel = starts[b0 : b0 + batch]
        frames = torch.stack([x[:, s : s + C] for s in sel])
        model.forward_device(frames, out=out[b0 : b0 + len(sel)], check=False)
        if progress is not None:
            torch.cuda.current_stream(x.device).synchronize()
            progress(done0 + b0 + len(sel), total)
    if check:
        model.check()


def overlap_add_cuda(
    model,
    x: torch.Tensor,
    chunk: int,
    overlap: float,
    batch: int = 8,
    progress: Callable[[int, int], None] | None = None,
    check: bool = True,
) -> torch.Tensor:
    """Device overlap-add: x (2, n) float32 on the model's GPU -> (2, n) on the same GPU."""
    n = x.shape[1]
    C = min(chunk, n)
    starts = chunk_starts(n, C, step_for(C, overlap))
    L = model.output_length(C)
    outs = torch.empty(len(starts), 2, L, device=x.device, dtype=torch.float32)
    run_chunks(model, x, starts, C, batch, outs, progress, check=check)
    return ola_device(outs, starts, C, n)
