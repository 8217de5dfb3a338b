"""Chunk-parallel separation over the GPUs of one node (one process per GPU, torch.distributed).

A song's chunk list (the reference schedule, turbo_roformer/chunking.py:11-33) is split into contiguous
shards, one per rank. Each rank runs its shard through its own model replica in batched forwards; the
chunk outputs are then gathered to rank 0 in a single collective (NCCL over NVLink on GPUs, gloo on CPU
for tests), and rank 0 applies the Hamming overlap-add in start order, so the result equals the
single-device result bit for bit. There is no other collective.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

from .chunking import chunk_starts, hamming, step_for


def shard_bounds(n_chunks: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) chunk ranges; the first n_chunks % world ranks take one extra chunk."""
    q, r = divmod(n_chunks, world)
    out, lo = [], 0
    for k in range(world):
        hi = lo + q + (1 if k < r else 0)
        out.append((lo, hi))
        lo = hi
    return out


def gather_chunks(local: torch.Tensor, counts: list[int], group=None) -> torch.Tensor | None:
    """Single gather of per-rank chunk outputs (padded to the largest shard) to rank 0.

    local: (max_count, 2, L) on this rank (rows past this rank's count are ignored).
    Returns (sum(counts), 2, L) on rank 0, None elsewhere.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    gl = [torch.empty_like(local) for _ in range(world)] if rank == 0 else None
    dist.gather(local, gl, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([g[:c] for g, c in zip(gl, counts)], dim=0)


def separate_sharded(
    run_shard: Callable[[list[int], torch.Tensor], None],
    n: int,
    chunk: int,
    overlap: float,
    out_len: int,
    device: torch.device,
    ola: Callable[[torch.Tensor, list[int], int, int], torch.Tensor],
    group=None,
) -> torch.Tensor | None:
    """Generic sharded overlap-add.

    run_shard(starts, out): fill out[i] (2, out_len) with the model output of the chunk at starts[i].
    ola(chunks, starts, C, n): weighted overlap-add on rank 0.
    Returns (2, n) on rank 0, None on the other ranks.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    C = min(chunk, n)
    starts = chunk_starts(n, C, step_for(C, overlap))
    bounds = shard_bounds(len(starts), world)
    counts = [hi - lo for lo, hi in bounds]
    lo, hi = bounds[rank]
    local = torch.zeros(max(counts), 2, out_len, device=device, dtype=torch.float32)
    if hi > lo:
        run_shard(starts[lo:hi], local)
    allc = gather_chunks(local, counts, group)
    if rank != 0:
        return None
    return ola(allc, starts, C, n)


def shard_span(starts: list[int], chunk: int, lo: int, hi: int) -> tuple[int, int]:
    """Sample range [a, b) that the chunks lo..hi-1 of ``starts`` read (empty for an empty shard)."""
    return (starts[lo], starts[hi - 1] + chunk) if hi > lo else (0, 0)


def separate_from_host(
    mix: torch.Tensor,
    chunk: int,
    overlap: float,
    run_span: Callable[[torch.Tensor, list[int], torch.Tensor], None],
    out_len: int,
    device: torch.device,
    ola: Callable[[torch.Tensor, list[int], int, int], torch.Tensor],
    peak_limit: float = 0.9,
    group=None,
    out: torch.Tensor | None = None,
    post_stream: "torch.cuda.Stream | None" = None,
) -> torch.Tensor | None:
    """Sharded separation of one song held in host memory (separator.py:188-201 over the ranks).

    mix: (2, n) float32 on the CPU (pinned, for asynchronous copies), n >= chunk. Each rank copies only
    the samples its shard of chunks reads, the song's peak is max-reduced over the ranks (one scalar),
    the span is scaled by the peak gain min(1, peak_limit / peak), ``run_span(span, starts_in_span,
    local)`` fills local[i] with the output of the chunk at span[:, s : s + chunk], the outputs are
    gathered to rank 0, which runs the overlap-add, divides by the gain and copies the result into
    ``out`` (if given, asynchronously) or returns it on its device. Other ranks return None.

    ``post_stream`` (CUDA): the gather, overlap-add and copy back run there, after this song's forwards,
    so rank 0's next song can start computing while this one's result is assembled and copied out.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    n = mix.shape[1]
    if mix.ndim != 2 or mix.shape[0] != 2 or n < chunk:
        raise ValueError("mix must be (2, n) with n >= chunk (short clips: Separator.separate)")
    starts = chunk_starts(n, chunk, step_for(chunk, overlap))
    bounds = shard_bounds(len(starts), world)
    counts = [hi - lo for lo, hi in bounds]
    lo, hi = bounds[rank]
    a, b = shard_span(starts, chunk, lo, hi)
    span = torch.empty(2, b - a, device=device, dtype=torch.float32)
    for c in range(2):  # one contiguous copy per channel row
        span[c].copy_(mix[c, a:b], non_blocking=True)
    peak = span.abs().amax() if b > a else torch.zeros((), device=device)
    dist.all_reduce(peak, op=dist.ReduceOp.MAX, group=group)
    gain = torch.where(peak > peak_limit, (peak_limit / peak.double()).float(), torch.ones((), device=device))
    span.mul_(gain)
    local = torch.zeros(max(counts), 2, out_len, device=device, dtype=torch.float32)
    if hi > lo:
        run_span(span, [s - a for s in starts[lo:hi]], local)
    if post_stream is None:
        return _gather_ola(local, counts, starts, chunk, n, gain, ola, group, out, rank)
    post_stream.wait_stream(torch.cuda.current_stream(device))
    local.record_stream(post_stream)  # the allocator must not reuse it before the gather has read it
    gain.record_stream(post_stream)
    with torch.cuda.stream(post_stream):
        return _gather_ola(local, counts, starts, chunk, n, gain, ola, group, out, rank)


def _gather_ola(local, counts, starts, chunk, n, gain, ola, group, out, rank):
    allc = gather_chunks(local, counts, group)
    if rank != 0:
        return None
    inst = ola(allc, starts, chunk, n).div_(gain)
    if out is None:
        return inst
    out.copy_(inst, non_blocking=True)
    return out


def ola_torch(chunks: torch.Tensor, starts: list[int], C: int, n: int) -> torch.Tensor:
    """Overlap-add in torch (any device), start order, used by the CPU (gloo) path."""
    w = torch.from_numpy(hamming(C)).to(chunks.device)
    result = torch.zeros(2, n, dtype=torch.float32, device=chunks.device)
    weight = torch.zeros(n, dtype=torch.float32, device=chunks.device)
    L = min(C, chunks.shape[-1])
    for y, s in zip(chunks, starts):
        result[:, s : s + L] += y[:, :L] * w[:L]
        weight[s : s + L] += w[:L]
    return result.div_(weight.clamp_(min=1e-10))


def separate_song_cuda(sep, x: torch.Tensor, overlap: float = 2.0, group=None,
                       check: bool = True) -> torch.Tensor | None:
    """Shard one song over the process group with CUDA models.

    sep: a ``Separator`` (backend cuda) on this rank's GPU; x: (2, n) padded, gain-applied song on that GPU.
    Returns the (2, n) instrumental on rank 0's GPU, None elsewhere. ``check=False`` leaves the
    device-error check (a stream synchronisation) to the caller (``sep.net.check()``), so the host can
    queue the next song while the GPU works.
    """
    from .chunking import ola_device, run_chunks

    model = sep.net
    C = min(sep.chunk, x.shape[1])

    def run_shard(starts, out):
        run_chunks(model, x, starts, C, sep.batch, out, check=check)

    return separate_sharded(run_shard, x.shape[1], sep.chunk, overlap, model.output_length(C), x.device,
                            lambda ch, st, c, n: ola_device(ch, st, c, n), group)


def separate_song_from_host(sep, mix: torch.Tensor, overlap: float = 2.0, out: torch.Tensor | None = None,
                            group=None) -> torch.Tensor | None:
    """``separate_from_host`` with the ranks' CUDA models: mix (2, n) pinned float32 on the CPU, n >= the
    Separator's chunk; rank 0 gets the (2, n) instrumental (in ``out``, pinned, when given). Work is
    queued without a host synchronisation; the gather and overlap-add run on a second stream of the
    Separator, so synchronise the device (not just the current stream) before reading ``out``;
    ``sep.net.check()`` reports device-side errors."""
    from .chunking import ola_device, run_chunks

    model = sep.net
    C = sep.chunk

    def run_span(span, starts, local):
        run_chunks(model, span, starts, C, sep.batch, local, check=False)

    if getattr(sep, "_post_stream", None) is None:
        sep._post_stream = torch.cuda.Stream(model.device)
    return separate_from_host(mix, C, overlap, run_span, model.output_length(C), model.device,
                              lambda ch, st, c, n: ola_device(ch, st, c, n), group=group, out=out,
                              post_stream=sep._post_stream)
