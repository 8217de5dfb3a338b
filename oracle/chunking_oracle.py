"""CPU oracle for the chunk schedule and Hamming overlap-add.  TEST INFRASTRUCTURE ONLY.

Restates LoggeL/turbo-roformer ``src/turbo_roformer/chunking.py:11-61`` and the short-clip padding
and peak-gain handling of ``src/turbo_roformer/separator.py:188-201`` with numpy float32 arithmetic:
every weighted chunk is rounded to float32 before it is added (a multiply, then an add, each rounded),
chunks are added in start order, and the sum is divided by the summed window clamped at 1e-10. Those
are the reference loop's floating-point steps, so this oracle reproduces its output bit for bit. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.

Parity pin: ``tests/test_chunking.py`` checks it against the reference's own exact-value tests
(the 29-chunk 4:12 schedule, Hamming == numpy, identity reconstruction), and ``tests/test_oracle_golden.py``
against outputs of the reference's ``Separator`` stored in ``tests/golden/``.
"""

from __future__ import annotations

import numpy as np
import torch

PEAK = 0.9
_EPS = np.float32(1e-10)


def chunk_starts(n: int, chunk: int, step: int) -> list[int]:
    """Offsets 0, step, 2 step, ... whose chunk ends before n, then one chunk ending exactly at n
    (chunking.py:11-21). The end chunk is added only if some offset of the grid reaches it."""
    grid = range(0, n, step)
    inside = [o for o in grid if o + chunk < n]
    if len(inside) == len(grid):
        return inside
    end = max(n - chunk, 0)
    return inside if inside and inside[-1] == end else inside + [end]


def hamming(n: int) -> np.ndarray:
    """Symmetric Hamming window, float64 math rounded once to float32 (chunking.py:24-28)."""
    if n == 1:
        return np.ones(1, np.float32)
    phase = (2 * np.pi) * np.arange(n) / (n - 1)
    return (0.54 - 0.46 * np.cos(phase)).astype(np.float32)


def step_for(chunk: int, overlap: float) -> int:
    """Hop between chunk starts: floor(chunk / overlap), at least 1 and at most chunk (chunking.py:31-33)."""
    return min(max(int(chunk / overlap), 1), chunk)


class _Accumulator:
    """Hamming-weighted sums of chunk outputs and of the window, float32, in the order chunks arrive."""

    def __init__(self, n: int, C: int):
        self.win = hamming(C)
        self.num = np.zeros((2, n), np.float32)
        self.den = np.zeros(n, np.float32)
        self.C = C

    def add(self, start: int, y) -> None:
        y = np.asarray(torch.as_tensor(y).detach().cpu().float())
        k = min(self.C, y.shape[-1])
        w = self.win[:k]
        self.num[:, start : start + k] += y[:, :k] * w
        self.den[start : start + k] += w

    def result(self) -> torch.Tensor:
        return torch.from_numpy(self.num / np.maximum(self.den, _EPS))


def overlap_add(x: torch.Tensor, chunk: int, overlap: float, run) -> torch.Tensor:
    """x (2, n) -> (2, n): each chunk x[:, s:s+C] goes through ``run`` as (1, 2, C); the outputs' first
    min(C, L) samples are Hamming-weighted, summed and divided by the summed window (chunking.py:36-61)."""
    n = x.shape[1]
    C = min(chunk, n)
    acc = _Accumulator(n, C)
    for s in chunk_starts(n, C, step_for(C, overlap)):
        acc.add(s, run(x[:, s : s + C].unsqueeze(0).contiguous())[0])
    return acc.result()


def ola_from_outputs(ys: list[torch.Tensor], starts: list[int], n: int, C: int) -> torch.Tensor:
    """The same overlap-add given precomputed chunk outputs ys[i] (2, L_i) in start order."""
    acc = _Accumulator(n, C)
    for s, y in zip(starts, ys):
        acc.add(s, y)
    return acc.result()


def separate_44k(x: np.ndarray, chunk: int, hop: int, overlap: float, run) -> np.ndarray:
    """The separator's 44.1 kHz path (separator.py:188-201): a clip shorter than a chunk that is not
    whole hops, or under 3 hops, is zero-padded to whole hops (at least 3); the mix is scaled to peak 0.9
    when louder; overlap-add; the scale undone; the padding trimmed."""
    n0 = x.shape[1]
    if n0 < chunk and (n0 % hop or n0 < 3 * hop):
        padded = np.zeros((x.shape[0], max(-(-n0 // hop), 3) * hop), x.dtype)
        padded[:, :n0] = x
        x = padded
    peak = float(np.abs(x).max())
    gain = PEAK / peak if peak > PEAK else 1.0
    scaled = x * np.float32(gain) if gain != 1.0 else x
    inst = overlap_add(torch.from_numpy(np.ascontiguousarray(scaled)), chunk, overlap, run)
    if gain != 1.0:
        inst.div_(gain)
    return np.ascontiguousarray(inst.numpy()[:, :n0])
