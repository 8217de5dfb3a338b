"""CPU oracle for the chunk schedule and Hamming overlap-add.  TEST INFRASTRUCTURE ONLY.

Restates LoggeL/turbo-roformer ``src/turbo_roformer/chunking.py:11-61`` and the short-clip padding
and peak-gain handling of ``src/turbo_roformer/separator.py:188-201``. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.

Parity pin: ``tests/test_chunking.py`` checks it against the reference's own exact-value tests
(the 29-chunk 4:12 schedule, Hamming == numpy, identity reconstruction).
"""

from __future__ import annotations

import numpy as np
import torch

PEAK = 0.9


def chunk_starts(n: int, chunk: int, step: int) -> list[int]:
    """Regular steps; the tail chunk is aligned to the end of the signal (chunking.py:11-21)."""
    starts: list[int] = []
    for off in range(0, n, step):
        if off + chunk >= n:
            tail = max(n - chunk, 0)
            if not starts or starts[-1] != tail:
                starts.append(tail)
            break
        starts.append(off)
    return starts


def hamming(n: int) -> np.ndarray:
    """Symmetric Hamming window 0.54 - 0.46 cos(2 pi k / (n - 1)) in float32 (chunking.py:24-28)."""
    if n == 1:
        return np.ones(1, np.float32)
    return (0.54 - 0.46 * np.cos(2 * np.pi * np.arange(n) / (n - 1))).astype(np.float32)


def step_for(chunk: int, overlap: float) -> int:
    """step = floor(chunk / overlap), clamped to [1, chunk] (chunking.py:31-33)."""
    return max(1, min(chunk, int(chunk / overlap)))


def overlap_add(x: torch.Tensor, chunk: int, overlap: float, run) -> torch.Tensor:
    """x (2, n) -> (2, n): Hamming-weighted sum of chunk predictions / summed weights (chunking.py:36-61)."""
    n = x.shape[1]
    C = min(chunk, n)
    starts = chunk_starts(n, C, step_for(C, overlap))
    w = torch.from_numpy(hamming(C))
    result = torch.zeros(2, n, dtype=torch.float32)
    weight = torch.zeros(n, dtype=torch.float32)
    for s in starts:
        y = run(x[:, s : s + C].unsqueeze(0).contiguous())[0]
        L = min(C, y.shape[-1])
        result[:, s : s + L] += y[:, :L].float() * w[:L]
        weight[s : s + L] += w[:L]
    return result.div_(weight.clamp_(min=1e-10))


def ola_from_outputs(ys: list[torch.Tensor], starts: list[int], n: int, C: int) -> torch.Tensor:
    """The same overlap-add given precomputed chunk outputs ys[i] (2, L_i) in start order."""
    w = torch.from_numpy(hamming(C))
    result = torch.zeros(2, n, dtype=torch.float32)
    weight = torch.zeros(n, dtype=torch.float32)
    for y, s in zip(ys, starts):
        L = min(C, y.shape[-1])
        result[:, s : s + L] += y[:, :L].float() * w[:L]
        weight[s : s + L] += w[:L]
    return result.div_(weight.clamp_(min=1e-10))


def separate_44k(x: np.ndarray, chunk: int, hop: int, overlap: float, run) -> np.ndarray:
    """Short-clip padding, peak gain to 0.9, overlap-add, undo gain, trim (separator.py:188-201)."""
    n0 = x.shape[1]
    if n0 < chunk and (n0 % hop or n0 < 3 * hop):
        target = max(-(-n0 // hop) * hop, 3 * hop)
        x = np.pad(x, ((0, 0), (0, target - n0)))
    peak = float(np.abs(x).max())
    gain = PEAK / peak if peak > PEAK else 1.0
    xt = torch.from_numpy(np.ascontiguousarray(x * np.float32(gain) if gain != 1.0 else x))
    inst = overlap_add(xt, chunk, overlap, run)
    if gain != 1.0:
        inst.div_(gain)
    return np.ascontiguousarray(inst.numpy()[:, :n0])
