"""trc_ola_noalloc, the overlap-add for callers that cannot allocate device memory while they run (an
audio plugin whose host application owns the device memory, a real-time audio thread that must not block
in the allocator). Its output must equal the allocating trc_ola exactly (the overlap-add is
bit-identical to the reference), on two calls in a row, because every call reuses the same fixed
staging arrays inside the library; it must not allocate; and a repeat call with an unchanged chunk
length must not re-upload the window. This file is named to be collected last."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

CU_MEMPOOL_ATTR_USED_MEM_HIGH = 8  # cuda.h CUmemPool_attribute


def _ola(lib, fn, chunks, starts, chunk, n, sync=True, out=None):
    from turbo_roformer_b200 import _lib

    if out is None:
        out = torch.full((2, n), float("nan"), device=chunks.device)
    st = (ctypes.c_int64 * len(starts))(*starts)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(getattr(lib, fn)(ctypes.c_void_p(chunks.data_ptr()), chunks.shape[2], st, len(starts), chunk, n,
                                ctypes.c_void_p(out.data_ptr()), stream))
    if sync:
        torch.cuda.synchronize()
    return out


def _case(seed, n, chunk, hop, overlap):
    from turbo_roformer_b200.chunking import chunk_starts, step_for

    g = torch.Generator().manual_seed(seed)
    starts = chunk_starts(n, chunk, step_for(chunk, overlap))
    clen = hop * (chunk // hop)
    chunks = torch.randn(len(starts), 2, clen, generator=g).cuda()
    return chunks, starts


class _DefaultPool:
    """The device's default memory pool (the one cudaMallocAsync draws from), through the driver API."""

    def __init__(self, device: int):
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.pool = ctypes.c_void_p()
        dev = ctypes.c_int()
        assert self.cu.cuDeviceGet(ctypes.byref(dev), device) == 0
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), dev) == 0

    def reset_high(self):
        zero = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolSetAttribute(self.pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH, ctypes.byref(zero)) == 0

    def high(self) -> int:
        v = ctypes.c_uint64(0)
        assert self.cu.cuMemPoolGetAttribute(self.pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH, ctypes.byref(v)) == 0
        return v.value


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


def test_noalloc_ola_allocates_nothing(cuda_device):
    """Neither the stream-ordered pool nor cudaMalloc grows during the calls (the allocating entry point
    shows that the pool check can tell the two apart)."""
    from turbo_roformer_b200 import _lib

    lib = _lib.load(build_if_missing=False)
    chunks, starts = _case(3, 1_000_000, 16_256, 128, 2.0)
    _ola(lib, "trc_ola_noalloc", chunks, starts, 16_256, 1_000_000)  # set-up for this context
    outs = [torch.empty(2, 1_000_000, device="cuda") for _ in range(3)]
    pool = _DefaultPool(torch.cuda.current_device())
    pool.reset_high()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for out in outs:
        _ola(lib, "trc_ola_noalloc", chunks, starts, 16_256, 1_000_000, out=out)
    free1, _ = torch.cuda.mem_get_info()
    assert pool.high() == 0
    assert free1 == free0
    _ola(lib, "trc_ola", chunks, starts, 16_256, 1_000_000)
    assert pool.high() > 0


def test_noalloc_ola_repeat_call_skips_the_window_upload(cuda_device):
    """With the window already on the device, a call returns while the stream is still busy and counts
    exactly one kernel launch; the result stays exact."""
    from turbo_roformer_b200 import _lib

    lib = _lib.load(build_if_missing=False)
    lib.trc_launch_count.restype = ctypes.c_longlong
    n, chunk = 2_000_000, 749_259
    chunks, starts = _case(4, n, chunk, 441, 2.0)
    ref = _ola(lib, "trc_ola", chunks, starts, chunk, n)
    _ola(lib, "trc_ola_noalloc", chunks, starts, chunk, n)  # uploads this chunk length's window
    busy_s = 0.5
    torch.cuda._sleep(int(busy_s * 2.0e9))  # keeps the stream busy for about busy_s or longer
    launches0 = lib.trc_launch_count()
    t0 = time.perf_counter()
    got = _ola(lib, "trc_ola_noalloc", chunks, starts, chunk, n, sync=False)
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    assert lib.trc_launch_count() - launches0 == 1
    assert host_s < 0.2 * busy_s, f"the repeat call blocked the host for {host_s * 1e3:.1f} ms"
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
