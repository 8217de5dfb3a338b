"""trc_ola_noalloc, the overlap-add for callers that cannot allocate device memory while they run (an
audio plugin whose host application owns the device memory, a real-time audio thread that must not block
in the allocator). Its output must equal the allocating trc_ola exactly (the overlap-add is
bit-identical to the reference), on two calls in a row, because every call reuses the same fixed
staging arrays inside the library. This file is named to be collected last."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ola(lib, fn, chunks, starts, chunk, n):
    from turbo_roformer_b200 import _lib

    out = torch.full((2, n), float("nan"), device=chunks.device)
    st = (ctypes.c_int64 * len(starts))(*starts)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(getattr(lib, fn)(ctypes.c_void_p(chunks.data_ptr()), chunks.shape[2], st, len(starts), chunk, n,
                                ctypes.c_void_p(out.data_ptr()), stream))
    torch.cuda.synchronize()
    return out


def _case(seed, n, chunk, hop, overlap):
    from turbo_roformer_b200.chunking import chunk_starts, step_for

    g = torch.Generator().manual_seed(seed)
    starts = chunk_starts(n, chunk, step_for(chunk, overlap))
    clen = hop * (chunk // hop)
    chunks = torch.randn(len(starts), 2, clen, generator=g).cuda()
    return chunks, starts


def test_noalloc_ola_equals_allocating_ola_twice(cuda_device):
    from turbo_roformer_b200 import _lib

    lib = _lib.load(build_if_missing=False)
    # two calls in a row with different sizes: the second must not see the first call's window/starts
    for seed, n, chunk, hop, overlap in ((1, 2_000_000, 749_259, 441, 2.0), (2, 300_000, 16_256, 128, 3.0)):
        chunks, starts = _case(seed, n, chunk, hop, overlap)
        ref = _ola(lib, "trc_ola", chunks, starts, chunk, n)
        got = _ola(lib, "trc_ola_noalloc", chunks, starts, chunk, n)
        assert torch.isfinite(ref).all()
        torch.testing.assert_close(got, ref, rtol=0, atol=0)


def test_noalloc_ola_rejects_sizes_beyond_its_arrays(cuda_device):
    from turbo_roformer_b200 import _lib

    lib = _lib.load(build_if_missing=False)
    too_long = (1 << 21) + 1
    st = (ctypes.c_int64 * 1)(0)
    dummy = torch.zeros(1, 2, 8, device="cuda")
    rc = lib.trc_ola_noalloc(ctypes.c_void_p(dummy.data_ptr()), 8, st, 1, too_long, too_long,
                             ctypes.c_void_p(dummy.data_ptr()), None)
    assert rc == -1 and b"TRC_OLA_NOALLOC_MAX_CHUNK" in lib.trc_last_error()
    many = 8193
    st = (ctypes.c_int64 * many)(*range(many))
    rc = lib.trc_ola_noalloc(ctypes.c_void_p(dummy.data_ptr()), 1, st, many, 1, many,
                             ctypes.c_void_p(dummy.data_ptr()), None)
    assert rc == -1 and b"TRC_OLA_NOALLOC_MAX_CHUNKS" in lib.trc_last_error()
