"""Per-kernel parity through the C ABI: each sm_100a stage against the CPU oracle's math on the same inputs.

fp32 stages (STFT, band split, norm, iSTFT) are held to >= 100 dB; 16-bit tensor-core stages (fp16
operands, fp32 accumulation) to >= 50 dB against fp32 math on the same 16-bit-rounded inputs. Shapes
cover partial tiles (T not a multiple of 128), batches > 1, and both attention modes.
"""

from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

from oracle import roformer_oracle as R

from .conftest import snr_db

pytestmark = pytest.mark.gpu


def vp(t: torch.Tensor) -> ctypes.c_void_p:
    """Raw device pointer; the caller keeps `t` alive (a temporary would return to torch's cache)."""
    return ctypes.c_void_p(t.data_ptr())


def stream(m) -> ctypes.c_void_p:
    return ctypes.c_void_p(m.stream_ptr())


def call(m, name, *args):
    from turbo_roformer_b200 import _lib

    _lib.check(getattr(m.lib, name)(m.handle, *args))
    m.check()


def layer_prefix(layer: int) -> str:
    return f"layers.{layer // 2}.{layer % 2}.layers.0."


def fold_qkv(sd, layer):
    p = layer_prefix(layer)
    g = sd[p + "0.norm.gamma"] * 16.0
    W = sd[p + "0.to_qkv.weight"] * g[None, :]
    W[:512] *= 0.125
    Wg = sd[p + "0.to_gates.weight"] * g[None, :]
    return W, Wg, sd[p + "0.to_gates.bias"]


def to_sequences(x, B, T, Fb, mode):
    """x (B*T*F, 8*64) per-token heads -> (sequences, L, 64) in the kernel's attention layout."""
    x = x.view(B, T, Fb, 8, 64)
    if mode == 0:
        return x.permute(0, 2, 3, 1, 4).reshape(B * Fb * 8, T, 64)
    return x.permute(0, 1, 3, 2, 4).reshape(B * T * 8, Fb, 64)


def from_sequences(o, B, T, Fb, mode):
    """(sequences, L, 64) -> (B*T*F, 8*64)"""
    if mode == 0:
        return o.view(B, Fb, 8, T, 64).permute(0, 3, 1, 2, 4).reshape(B * T * Fb, 512)
    return o.view(B, T, 8, Fb, 64).permute(0, 1, 3, 2, 4).reshape(B * T * Fb, 512)


# ------------------------------------------------------------------------------------------------ fp32 stages
@pytest.mark.parametrize("B,n", [(1, 16256), (2, 5000)])
def test_stft_matches_oracle(tiny_cuda, tiny_cfg, B, n):
    g = torch.Generator().manual_seed(n)
    audio = torch.randn(B, 2, n, generator=g) * 0.3
    _, xin_ref = R.stft(audio, tiny_cfg)
    T = xin_ref.shape[1]
    xin = torch.empty(B, T, 4 * tiny_cfg.n_freqs, device="cuda")
    audio_d = audio.cuda()
    call(tiny_cuda, "trc_stft", vp(audio_d), B, n, vp(xin), stream(tiny_cuda))
    assert snr_db(xin_ref.numpy(), xin.cpu().numpy()) >= 100.0


@pytest.mark.parametrize("B,T", [(2, 77), (1, 300)])
def test_band_split_matches_oracle(tiny_cuda, tiny_cfg, tiny_sd, B, T):
    """Band split as one grouped tensor-core GEMM over the bands: each band's inputs are L2-normalised
    and rounded to fp16, the folded weights are fp16, accumulation is fp32; held to the 16-bit stages'
    50 dB against the fp32 oracle (and against fp32 math on the same rounded operands it is exact to
    accumulation order)."""
    g = torch.Generator().manual_seed(1 + T)
    xin = torch.randn(B, T, 4 * tiny_cfg.n_freqs, generator=g) * torch.logspace(-3, 1, 4 * tiny_cfg.n_freqs)
    ref = R.band_split(xin, tiny_sd, tiny_cfg).reshape(B * T * tiny_cfg.n_bands, 256)
    X = torch.empty(B * T * tiny_cfg.n_bands, 256, device="cuda")
    xin_d = xin.cuda()
    call(tiny_cuda, "trc_band_split", vp(xin_d), B, T, vp(X), stream(tiny_cuda))
    assert snr_db(ref.numpy(), X.cpu().numpy()) >= 50.0
    # fp32 math on the fp16-rounded normalised inputs and weights: only the accumulation order differs
    parts, outs = xin.split(tiny_cfg.band_dims, dim=-1), []
    for k, part in enumerate(parts):
        p = f"band_split.to_features.{k}."
        xn = (part / part.norm(dim=-1, keepdim=True).clamp_min(1e-12)).half().float()
        w = (tiny_sd[p + "1.weight"] * (part.shape[-1] ** 0.5) * tiny_sd[p + "0.gamma"][None, :]).half().float()
        outs.append(xn @ w.T + tiny_sd[p + "1.bias"])
    ref16 = torch.stack(outs, dim=-2).reshape(B * T * tiny_cfg.n_bands, 256)
    assert snr_db(ref16.numpy(), X.cpu().numpy()) >= 100.0


def test_add_rmsnorm(tiny_cuda):
    rows = 1000
    X = torch.randn(rows, 256)
    Y = torch.randn(rows, 256)
    ref = X + Y
    ref_n = F.normalize(ref, dim=-1)
    Xd, Yd = X.cuda(), Y.cuda()
    out = torch.empty(rows, 256, device="cuda")
    call(tiny_cuda, "trc_add_rmsnorm", vp(Xd), vp(Yd), vp(out), 1, rows, ctypes.c_float(1e-12), stream(tiny_cuda))
    assert snr_db(ref.numpy(), Xd.cpu().numpy()) >= 140.0
    assert snr_db(ref_n.numpy(), out.cpu().numpy()) >= 130.0
    out16 = torch.empty(rows, 256, device="cuda", dtype=torch.float16)
    call(tiny_cuda, "trc_add_rmsnorm", vp(Xd), None, vp(out16), 0, rows, ctypes.c_float(1e-12), stream(tiny_cuda))
    assert snr_db(ref_n.numpy(), out16.float().cpu().numpy()) >= 65.0


def test_istft_matches_oracle(tiny_cuda, tiny_cfg):
    B, n = 2, 16256
    g = torch.Generator().manual_seed(3)
    audio = torch.randn(B, 2, n, generator=g) * 0.3
    spec, xin = R.stft(audio, tiny_cfg)
    T = xin.shape[1]
    mask = torch.randn(B, T, 4 * tiny_cfg.n_freqs, generator=g)
    ref = R.istft_apply(spec, mask, tiny_cfg)
    out = torch.empty(B, 2, tiny_cfg.stft_hop_length * (T - 1), device="cuda")
    frames = torch.empty(B * T * 2 * tiny_cfg.stft_n_fft, device="cuda")
    xin_d, mask_d = xin.cuda(), mask.cuda()
    call(tiny_cuda, "trc_istft", vp(xin_d), vp(mask_d), B, T, vp(out), vp(frames), stream(tiny_cuda))
    assert out.shape == ref.shape
    assert snr_db(ref.numpy(), out.cpu().numpy()) >= 100.0


# ------------------------------------------------------------------------------------------------ tensor-core stages
@pytest.mark.parametrize("layer", [0, 1, 3])
@pytest.mark.parametrize("B,T", [(1, 128), (2, 77)])
def test_qkv_rope_gemm(tiny_cuda, tiny_cfg, tiny_sd, layer, B, T):
    Fb = tiny_cfg.n_bands
    N = B * T * Fb
    mode = layer % 2
    g = torch.Generator().manual_seed(10 + layer)
    xn = F.normalize(torch.randn(N, 256, generator=g), dim=-1).half()
    W, Wg, bg = fold_qkv(tiny_sd, layer)
    ref = xn.float() @ torch.cat([W, Wg]).t()
    freqs = tiny_sd[layer_prefix(layer) + "0.rotary_embed.freqs"]
    q = R.rotate(to_sequences(ref[:, :512], B, T, Fb, mode), freqs)
    k = R.rotate(to_sequences(ref[:, 512:1024], B, T, Fb, mode), freqs)
    v = to_sequences(ref[:, 1024:1536], B, T, Fb, mode)
    gates = torch.sigmoid(ref[:, 1536:] + bg)
    Q = torch.empty(N * 512, device="cuda", dtype=torch.float16)
    K, V = torch.empty_like(Q), torch.empty_like(Q)
    G = torch.empty(N, 8, device="cuda")
    xn_d = xn.cuda()
    call(tiny_cuda, "trc_qkv_rope_gemm", layer, vp(xn_d), B, T, vp(Q), vp(K), vp(V), vp(G), stream(tiny_cuda))
    assert snr_db(q.numpy(), Q.view_as(q).float().cpu().numpy()) >= 50.0
    assert snr_db(k.numpy(), K.view_as(k).float().cpu().numpy()) >= 50.0
    assert snr_db(v.numpy(), V.view_as(v).float().cpu().numpy()) >= 50.0
    assert snr_db(gates.numpy(), G.cpu().numpy()) >= 60.0


def attention_ref(Q, K, V, G, B, T, Fb, mode, subset=None):
    q, k, v = Q.float(), K.float(), V.float()
    if subset is not None:
        q, k, v = q[subset], k[subset], v[subset]
    o = F.scaled_dot_product_attention(q, k, v, scale=1.0)
    return o


@pytest.mark.parametrize("mode,B,T", [(0, 1, 128), (0, 2, 77), (0, 1, 300), (1, 1, 128), (1, 2, 77)])
def test_attention(tiny_cuda, tiny_cfg, mode, B, T):
    Fb = tiny_cfg.n_bands
    N = B * T * Fb
    L = T if mode == 0 else Fb
    BH = N * 8 // L
    g = torch.Generator().manual_seed(100 * mode + T)
    Q = (torch.randn(BH, L, 64, generator=g) * 0.25).half()
    K = (torch.randn(BH, L, 64, generator=g) * 0.25).half()
    V = torch.randn(BH, L, 64, generator=g).half()
    G = torch.rand(N, 8, generator=g)
    o = attention_ref(Q, K, V, G, B, T, Fb, mode)
    ref = from_sequences(o, B, T, Fb, mode).view(N, 8, 64) * G[:, :, None]
    O = torch.empty(N, 512, device="cuda", dtype=torch.float16)
    Qd, Kd, Vd, Gd = Q.cuda(), K.cuda(), V.cuda(), G.cuda()
    call(tiny_cuda, "trc_attention", mode, vp(Qd), vp(Kd), vp(Vd), vp(Gd), vp(O), B, T, stream(tiny_cuda))
    assert snr_db(ref.reshape(N, 512).numpy(), O.float().cpu().numpy()) >= 50.0


@pytest.mark.parametrize("T", [1, 63, 64, 65, 129, 256, 257, 384, 385, 640, 700])
def test_attention_time_item_edges(tiny_cuda, tiny_cfg, T):
    """Time mode around the kernel's item and step edges: items of three 128-row query tiles (a last item
    with one, two or three tiles inside the sequence) and 64-key steps (a last step with 1..64 keys)."""
    B, Fb = 1, tiny_cfg.n_bands
    N = B * T * Fb
    BH = N * 8 // T
    g = torch.Generator().manual_seed(1000 + T)
    Q = (torch.randn(BH, T, 64, generator=g) * 0.25).half()
    K = (torch.randn(BH, T, 64, generator=g) * 0.25).half()
    V = torch.randn(BH, T, 64, generator=g).half()
    G = torch.rand(N, 8, generator=g)
    o = attention_ref(Q, K, V, G, B, T, Fb, 0)
    ref = from_sequences(o, B, T, Fb, 0).view(N, 8, 64) * G[:, :, None]
    O = torch.full((N, 512), float("nan"), device="cuda", dtype=torch.float16)
    Qd, Kd, Vd, Gd = Q.cuda(), K.cuda(), V.cuda(), G.cuda()
    call(tiny_cuda, "trc_attention", 0, vp(Qd), vp(Kd), vp(Vd), vp(Gd), vp(O), B, T, stream(tiny_cuda))
    got = O.float().cpu()
    assert torch.isfinite(got).all()  # every output row written
    assert snr_db(ref.reshape(N, 512).numpy(), got.numpy()) >= 50.0


def test_attention_full_length(tiny_cuda, tiny_cfg):
    """Time attention over T = 1701 frames (14 key tiles, ragged last tile), a subset of sequences checked."""
    B, T, Fb = 1, 1701, tiny_cfg.n_bands
    N = B * T * Fb
    BH = Fb * 8
    g = torch.Generator().manual_seed(7)
    Q = (torch.randn(BH, T, 64, generator=g) * 0.3).half()
    K = (torch.randn(BH, T, 64, generator=g) * 0.3).half()
    V = torch.randn(BH, T, 64, generator=g).half()
    G = torch.rand(N, 8, generator=g)
    O = torch.empty(N, 512, device="cuda", dtype=torch.float16)
    Qd, Kd, Vd, Gd = Q.cuda(), K.cuda(), V.cuda(), G.cuda()
    call(tiny_cuda, "trc_attention", 0, vp(Qd), vp(Kd), vp(Vd), vp(Gd), vp(O), B, T, stream(tiny_cuda))
    subset = torch.arange(0, BH, 13)
    o = attention_ref(Q, K, V, G, B, T, Fb, 0, subset)
    Ok = O.float().cpu().view(T, Fb, 8, 64)
    for i, bh in enumerate(subset.tolist()):
        f, h = bh // 8, bh % 8
        ref = o[i] * G.view(T, Fb, 8)[:, f, h, None]
        assert snr_db(ref.numpy(), Ok[:, f, h].numpy()) >= 50.0, bh


@pytest.mark.parametrize("which", [0, 1])
def test_gemm_res_norm(tiny_cuda, tiny_cfg, tiny_sd, which):
    layer = 2
    B, T = 1, 77
    N = B * T * tiny_cfg.n_bands
    p = layer_prefix(layer)
    g = torch.Generator().manual_seed(20 + which)
    if which == 0:
        A = (torch.randn(N, 512, generator=g) * 0.5).half()
        W, b = tiny_sd[p + "0.to_out.0.weight"], None
    else:
        A = (torch.randn(N, tiny_cfg.ff_inner, generator=g) * 0.5).half()
        W, b = tiny_sd[p + "1.net.4.weight"], tiny_sd[p + "1.net.4.bias"]
    X = torch.randn(N, 256, generator=g)
    y = A.float() @ W.t()
    if b is not None:
        y = y + b
    Xr = X + y
    xn_ref = F.normalize(Xr, dim=-1)
    Xd = X.cuda()
    xn = torch.empty(N, 256, device="cuda", dtype=torch.float16)
    Ad = A.cuda()
    call(tiny_cuda, "trc_gemm_res_norm", layer, which, vp(Ad), vp(Xd), vp(xn), N, stream(tiny_cuda))
    assert snr_db((Xr - X).numpy(), (Xd.cpu() - X).numpy()) >= 50.0  # the added GEMM term
    assert snr_db(xn_ref.numpy(), xn.float().cpu().numpy()) >= 55.0


@pytest.mark.parametrize("mode", [0, 1])
def test_rope_pack_matches_reference_semantics(tiny_cuda, tiny_cfg, tiny_sd, mode):
    """rope_pack (kernels.cpp:161-248, unpacked): rotary in fp32 on the 16-bit GEMM output, one rounding."""
    B, T = 2, 37
    Fb = tiny_cfg.n_bands
    N = B * T * Fb
    g = torch.Generator().manual_seed(30 + mode)
    qkvg = (torch.randn(N, 1544, generator=g) * 0.5).half()
    x = qkvg.float()
    freqs = tiny_sd[layer_prefix(mode) + "0.rotary_embed.freqs"]
    q = R.rotate(to_sequences(x[:, :512], B, T, Fb, mode), freqs)
    k = R.rotate(to_sequences(x[:, 512:1024], B, T, Fb, mode), freqs)
    v = to_sequences(qkvg[:, 1024:1536], B, T, Fb, mode)
    gates = torch.sigmoid(x[:, 1536:])
    Q = torch.empty(N * 512, device="cuda", dtype=torch.float16)
    K, V = torch.empty_like(Q), torch.empty_like(Q)
    G = torch.empty(N, 8, device="cuda")
    qd = qkvg.cuda()
    call(tiny_cuda, "trc_rope_pack", mode, vp(qd), B, T, vp(Q), vp(K), vp(V), vp(G), stream(tiny_cuda))
    # one fp32 rotation then one rounding: at most one 16-bit ulp from the rounded fp32 reference
    for ref, got in ((q, Q), (k, K)):
        got = got.view_as(ref).float().cpu()
        ulp = torch.finfo(torch.float16).eps * ref.abs().clamp(min=2**-14)
        assert ((got - ref).abs() <= ulp).all()
    assert torch.equal(V.view_as(v).cpu(), v)  # v is moved, not recomputed
    torch.testing.assert_close(G.cpu(), gates, rtol=2e-6, atol=2e-7)
    with pytest.raises(Exception):
        call(tiny_cuda, "trc_rope_pack", 2, vp(qd), B, T, vp(Q), vp(K), vp(V), vp(G), stream(tiny_cuda))


@pytest.mark.parametrize("mode", [0, 1])
def test_gate_merge_is_exact(tiny_cuda, tiny_cfg, mode):
    """gate_merge (kernels.cpp:391-408): O = gate * A per head, one fp32 product rounded once."""
    B, T = 2, 45
    Fb = tiny_cfg.n_bands
    N = B * T * Fb
    g = torch.Generator().manual_seed(40 + mode)
    L = T if mode == 0 else Fb
    A = torch.randn(N * 8 // L, L, 64, generator=g).half()
    G = torch.rand(N, 8, generator=g)
    O = torch.empty(N, 512, device="cuda", dtype=torch.float16)
    Ad, Gd = A.cuda(), G.cuda()
    call(tiny_cuda, "trc_gate_merge", mode, vp(Ad), vp(Gd), vp(O), B, T, stream(tiny_cuda))
    gate_seq = to_sequences(G.repeat_interleave(64, dim=1), B, T, Fb, mode)
    ref = from_sequences((A.float() * gate_seq).half(), B, T, Fb, mode)
    assert torch.equal(O.cpu(), ref)


@pytest.mark.parametrize("in_place", [False, True])
def test_ffn_res_norm_fused(tiny_cuda, tiny_cfg, tiny_sd, in_place):
    """Fused FF block == gemm_gelu then gemm_res_norm (kernels.cpp:610-642, :543-586) in fp32 math."""
    layer = 3
    B, T = 1, 91  # 2639 rows: a partial last 128-row block
    N = B * T * tiny_cfg.n_bands
    p = layer_prefix(layer)
    g = torch.Generator().manual_seed(50 + int(in_place))
    xn = F.normalize(torch.randn(N, 256, generator=g), dim=-1).half()
    X = torch.randn(N, 256, generator=g)
    gamma = tiny_sd[p + "1.net.0.gamma"]
    W1 = tiny_sd[p + "1.net.1.weight"] * (gamma * 16.0)[None, :]
    Hr = F.gelu(xn.float() @ W1.t() + tiny_sd[p + "1.net.1.bias"])
    y = Hr @ tiny_sd[p + "1.net.4.weight"].t() + tiny_sd[p + "1.net.4.bias"]
    Xr = X + y
    xn_ref = F.normalize(Xr, dim=-1)
    Xd, xd = X.cuda(), xn.cuda()
    out = xd if in_place else torch.empty_like(xd)
    call(tiny_cuda, "trc_ffn_res_norm", layer, vp(xd), vp(Xd), vp(out), N, stream(tiny_cuda))
    assert snr_db(y.numpy(), (Xd.cpu() - X).numpy()) >= 50.0  # the added feed-forward term
    assert snr_db(xn_ref.numpy(), out.float().cpu().numpy()) >= 55.0


def test_gemm_gelu(tiny_cuda, tiny_cfg, tiny_sd):
    layer = 1
    N = 2 * 77 * tiny_cfg.n_bands
    p = layer_prefix(layer)
    g = torch.Generator().manual_seed(30)
    xn = F.normalize(torch.randn(N, 256, generator=g), dim=-1).half()
    W1 = tiny_sd[p + "1.net.1.weight"] * (tiny_sd[p + "1.net.0.gamma"] * 16.0)[None, :]
    ref = F.gelu(xn.float() @ W1.t() + tiny_sd[p + "1.net.1.bias"])
    H = torch.empty(N, tiny_cfg.ff_inner, device="cuda", dtype=torch.float16)
    xn_d = xn.cuda()
    call(tiny_cuda, "trc_gemm_gelu", layer, vp(xn_d), vp(H), N, stream(tiny_cuda))
    assert snr_db(ref.numpy(), H.float().cpu().numpy()) >= 50.0


@pytest.mark.parametrize("B,T", [(1, 128), (2, 77)])
def test_mask_estimator(tiny_cuda, tiny_cfg, tiny_sd, B, T):
    Fb = tiny_cfg.n_bands
    N = B * T * Fb
    g = torch.Generator().manual_seed(40 + T)
    xn = F.normalize(torch.randn(N, 256, generator=g), dim=-1).half()
    x = xn.float().view(B, T, Fb, 256) * (tiny_sd["final_norm.gamma"] * 16.0)
    ref = R.mask_estimator(x, tiny_sd, tiny_cfg)
    mask = torch.empty(B, T, 4 * tiny_cfg.n_freqs, device="cuda")
    hid = torch.empty(Fb * B * T * tiny_cfg.mask_hidden, device="cuda", dtype=torch.float16)
    xn_d = xn.cuda()
    call(tiny_cuda, "trc_mask", vp(xn_d), B, T, vp(mask), vp(hid), stream(tiny_cuda))
    assert snr_db(ref.numpy(), mask.cpu().numpy()) >= 50.0
