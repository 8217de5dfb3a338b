"""The north star's isolated configurations at their stated shapes, through the C ABI.

* Config 2: one time-attention layer, Q/K/V [62 bands x 8 heads, 1701, 64] ~ N(0,1), rotary on Q and K
  with the fp32 tables, scale 1/8 folded into Q, 16-bit operands (fp16 and bf16 handles), against fp32
  SDPA on the unrounded inputs (the input-rounding floor shows here) and on the rounded inputs (kernel
  error alone). Reference kernel: turbo_roformer/csrc/kernels.cpp:255-388.
* The attention kernel's online-softmax rescale (a later key tile whose maximum exceeds the running
  maximum by more than 2^8), forced by a key ramp, against fp32 SDPA.
* Config 3: the 12-layer transformer stack alone (trc_transformer) on N(0,1) tokens [1701 x 62, 256]
  against the fp32 oracle's axial blocks (turbo_roformer/model.py:262-268; fast.py:259-266).

The fp32 attention reference runs in torch on the GPU (math backend, no TF32): a plain fp32 restatement
of the same op, as the per-kernel tests use.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from oracle import roformer_oracle as R
from turbo_roformer_b200 import synthetic as S

from .conftest import snr_db

pytestmark = pytest.mark.gpu

LOG2E = 1.4426950408889634
RESCALE_LOG2 = 8.0  # the kernel raises its running maximum only past this margin (log2 units)


def vp(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def full_handles(full_cfg, full_sd, cuda_device):
    from turbo_roformer_b200.backend import CudaBSRoformer

    return {p: CudaBSRoformer(full_sd, cfg=full_cfg, device=0, precision=p) for p in ("fp16", "bf16")}


def run_attention(m, Q, K, V, G, B, T, dtype):
    """trc_attention in time mode on device tensors; returns O (tokens, 512) as float32."""
    from turbo_roformer_b200 import _lib

    N = G.shape[0]
    O = torch.empty(N, 512, device="cuda", dtype=dtype)
    st = ctypes.c_void_p(m.stream_ptr())
    _lib.check(m.lib.trc_attention(m.handle, 0, vp(Q), vp(K), vp(V), vp(G), vp(O), B, T, st))
    m.check()
    return O.float()


def sdpa_fp32(q, k, v, chunk=32):
    """softmax(q k^T) v in fp32 (scale 1: the 1/8 is already in q), per group of sequences."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.empty_like(q, dtype=torch.float32)
        with sdpa_kernel(SDPBackend.MATH):
            for s in range(0, q.shape[0], chunk):
                out[s : s + chunk] = F.scaled_dot_product_attention(
                    q[s : s + chunk].float(), k[s : s + chunk].float(), v[s : s + chunk].float(), scale=1.0)
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def merge_time(o, G, T, Fb):
    """(Fb*8, T, 64) per-sequence outputs -> (T*Fb, 512) tokens, times the gates (time mode, batch 1)."""
    return (o.view(Fb, 8, T, 64).permute(2, 0, 1, 3).reshape(T * Fb, 8, 64) * G[:, :, None]).reshape(T * Fb, 512)


@pytest.mark.parametrize("precision", ["fp16", "bf16"])
def test_config2_time_attention_at_spec(full_handles, full_cfg, precision):
    T, Fb = 1701, full_cfg.n_bands
    BH = Fb * 8
    dtype = torch.float16 if precision == "fp16" else torch.bfloat16
    g = torch.Generator().manual_seed(0)
    q = torch.randn(BH, T, 64, generator=g)
    k = torch.randn(BH, T, 64, generator=g)
    v = torch.randn(BH, T, 64, generator=g)
    freqs = S.rotary_freqs(64)
    q = R.rotate(q, freqs) * 0.125  # dim_head ** -0.5, folded into Q (exact: a power of two)
    k = R.rotate(k, freqs)
    G = torch.ones(T * Fb, 8, device="cuda")
    qd, kd, vd = (t.to("cuda", dtype).contiguous() for t in (q, k, v))
    O = run_attention(full_handles[precision], qd, kd, vd, G, 1, T, dtype)
    ref_rounded = merge_time(sdpa_fp32(qd, kd, vd), G, T, Fb)
    ref_exact = merge_time(sdpa_fp32(q.cuda(), k.cuda(), v.cuda()), G, T, Fb)
    snr_kernel = snr_db(ref_rounded.cpu().numpy(), O.cpu().numpy())
    snr_total = snr_db(ref_exact.cpu().numpy(), O.cpu().numpy())
    floor = snr_db(ref_exact.cpu().numpy(), ref_rounded.cpu().numpy())
    print(f"config 2 [{BH}, {T}, 64] {precision}: {snr_kernel:.2f} dB vs fp32 SDPA on the rounded inputs, "
          f"{snr_total:.2f} dB vs fp32 SDPA on the unrounded inputs (input-rounding floor {floor:.2f} dB)")
    assert snr_kernel >= 50.0
    assert snr_total >= min(floor - 3.0, 50.0)  # kernel error no larger than the input rounding's


def _rescale_events(q, k, L, group=16):
    """Rows x key tiles where the kernel's online softmax must raise its running maximum (q, k: the
    16-bit inputs; scores in fp32, a group of sequences at a time)."""
    n_tiles = (L + 127) // 128
    total = 0
    for b in range(0, q.shape[0], group):
        s = torch.einsum("bid,bjd->bij", q[b : b + group].float(), k[b : b + group].float()) * LOG2E
        tile_max = torch.stack([s[:, :, 128 * t : min(L, 128 * t + 128)].amax(-1) for t in range(n_tiles)], -1)
        m_run = tile_max[..., 0].clone()
        for t in range(1, n_tiles):
            need = tile_max[..., t] > m_run + RESCALE_LOG2
            total += int(need.sum())
            m_run = torch.where(need, tile_max[..., t], m_run)
    return total


def test_attention_online_softmax_rescale(tiny_cuda, tiny_cfg):
    """Scores that rise along the keys (a ramp on one key dimension, seen by half of the query rows with a
    positive and half with a negative coefficient) plus a late spike: the running maximum must be raised
    many times, once by ~2^60, and the result still equals fp32 SDPA on the same rounded inputs."""
    T, Fb = 1701, tiny_cfg.n_bands
    BH = Fb * 8
    g = torch.Generator().manual_seed(5)
    q = torch.randn(BH, T, 64, generator=g) * 0.3
    k = torch.randn(BH, T, 64, generator=g) * 0.3
    v = torch.randn(BH, T, 64, generator=g)
    sign = torch.where(torch.arange(T) % 2 == 0, 3.0, -3.0)
    q[:, :, 0] = sign[None, :] + 0.1 * q[:, :, 0]
    k[:, :, 0] = torch.linspace(0.0, 12.0, T)[None, :]  # scores rise by ~36 nats over the keys for sign > 0
    k[:, 1500, 0] = 26.0  # a spike: +42 nats over the ramp at key 1500
    qd, kd, vd = (t.to("cuda", torch.float16).contiguous() for t in (q, k, v))
    events = _rescale_events(qd, kd, T)
    assert events > BH * T // 2 * 3  # every rising row rescales several times
    G = torch.rand(T * Fb, 8, generator=g).cuda()
    O = run_attention(tiny_cuda, qd, kd, vd, G, 1, T, torch.float16)
    ref = merge_time(sdpa_fp32(qd, kd, vd), G, T, Fb)
    snr = snr_db(ref.cpu().numpy(), O.cpu().numpy())
    print(f"rescale case: {events} rescale events, {snr:.2f} dB vs fp32 SDPA")
    assert torch.isfinite(O).all()
    assert snr >= 50.0


@pytest.mark.slow
def test_config3_transformer_stack(full_handles, full_cfg, full_sd):
    """Config 3: tokens [1701 x 62, 256] ~ N(0,1) (bf16-representable) through the 24 transformers. The
    output is compared whole and as the update the layers add to the input."""
    T, Fb, D = 1701, full_cfg.n_bands, full_cfg.dim
    g = torch.Generator().manual_seed(3)
    X0 = torch.randn(T * Fb, D, generator=g).to(torch.bfloat16).float()
    m = full_handles["fp16"]
    X = m.transformer_device(X0.cuda().contiguous(), 1, T).cpu()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    with torch.inference_mode():
        x = X0.view(1, T, Fb, D)
        for i in range(full_cfg.depth):
            x = R.axial_block(x, full_sd, full_cfg, i)
    ref = x.reshape(T * Fb, D)
    snr = snr_db(ref.numpy(), X.numpy())
    snr_update = snr_db((ref - X0).numpy(), (X - X0).numpy())
    print(f"config 3 stack: {snr:.2f} dB on the output, {snr_update:.2f} dB on the update the layers add")
    assert math.isfinite(snr) and snr >= 50.0
    assert snr_update >= 40.0
