"""CPU fp32 oracle for the BS-RoFormer forward.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker or the timed CPU baseline. The product (``turbo_roformer_b200``)
never imports it: its forward runs on the CUDA kernels or fails loudly.

It restates the reference's fp32 torch forward (LoggeL/turbo-roformer ``src/turbo_roformer/model.py``)
as plain functions over an upstream ``state_dict``, stage by stage, so that each CUDA kernel can be
checked against the stage it replaces. Every function cites the reference lines it follows.

Parity pin: ``tests/golden/make_golden.py`` runs the reference package itself (imported from its
source tree in the build container) on the same seeded weights and audio and stores the outputs
under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against them.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """``F.normalize(x) * sqrt(d) * gamma`` (model.py:28-35)."""
    return F.normalize(x, dim=-1) * (x.shape[-1] ** 0.5) * gamma


def rotary_angles(freqs: torch.Tensor, seq_len: int) -> torch.Tensor:
    """fp32 angles (seq, dim / 2): position times each pair's frequency (model.py:46-50)."""
    pos = torch.arange(seq_len, dtype=torch.float32)
    return pos[:, None] * freqs.float()[None, :]


def rotate(t: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Rotary embedding in fp32 on interleaved pairs (model.py:52-59): the pair (a, b) = (t[2i], t[2i+1])
    at position p becomes (a cos - b sin, b cos + a sin) with angle p * freqs[i]."""
    ang = rotary_angles(freqs, t.shape[-2])
    c, s = ang.cos(), ang.sin()
    tf = t.float()
    a, b = tf[..., 0::2], tf[..., 1::2]
    out = torch.empty_like(tf)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = b * c + a * s
    return out.to(t.dtype)


def attention(x: torch.Tensor, sd: dict, p: str, heads: int, dim_head: int) -> torch.Tensor:
    """Gated multi-head attention with rotary q/k (model.py:99-111). x (b, n, d) -> (b, n, d)."""
    b, n, _ = x.shape
    x = rmsnorm(x, sd[p + "norm.gamma"])
    qkv = F.linear(x, sd[p + "to_qkv.weight"])
    q, k, v = qkv.view(b, n, 3, heads, dim_head).permute(2, 0, 3, 1, 4)
    freqs = sd[p + "rotary_embed.freqs"]
    q = rotate(q, freqs)
    k = rotate(k, freqs)
    out = F.scaled_dot_product_attention(q, k, v)  # scale dim_head ** -0.5 (model.py:107)
    gates = F.linear(x, sd[p + "to_gates.weight"], sd[p + "to_gates.bias"])
    out = out * torch.sigmoid(gates).transpose(1, 2)[..., None]  # one gate per (head, position)
    out = out.transpose(1, 2).reshape(b, n, heads * dim_head)
    return F.linear(out, sd[p + "to_out.0.weight"])


def feedforward(x: torch.Tensor, sd: dict, p: str) -> torch.Tensor:
    """RMSNorm -> Linear -> GELU(erf) -> Linear (model.py:62-76)."""
    h = rmsnorm(x, sd[p + "net.0.gamma"])
    h = F.gelu(F.linear(h, sd[p + "net.1.weight"], sd[p + "net.1.bias"]))
    return F.linear(h, sd[p + "net.4.weight"], sd[p + "net.4.bias"])


def transformer(x: torch.Tensor, sd: dict, prefix: str, heads: int, dim_head: int) -> torch.Tensor:
    """Depth-1 transformer without output norm: x = attn(x) + x; x = ff(x) + x (model.py:140-144)."""
    x = attention(x, sd, prefix + "layers.0.0.", heads, dim_head) + x
    x = feedforward(x, sd, prefix + "layers.0.1.") + x
    return x


def stft(audio: torch.Tensor, cfg) -> tuple[torch.Tensor, torch.Tensor]:
    """audio (b, 2, L) fp32 -> (spec (b, 2F, T, 2) in "b (f s) t c" order, xin (b, T, 4F)) (model.py:251-260).

    Hann window (periodic), center=True reflect padding, onesided, not normalised (model.py:231-234).
    """
    b, s, t = audio.shape
    window = torch.hann_window(cfg.stft_win_length)
    spec = torch.view_as_real(
        torch.stft(
            audio.reshape(b * s, t),
            n_fft=cfg.stft_n_fft,
            hop_length=cfg.stft_hop_length,
            win_length=cfg.stft_win_length,
            normalized=False,
            window=window,
            return_complex=True,
        )
    )
    nf, nt = spec.shape[1], spec.shape[2]
    # (b s) f t c -> b (f s) t c: the two channels of a frequency bin become neighbouring rows
    spec = spec.reshape(b, s, nf, nt, 2).transpose(1, 2).reshape(b, nf * s, nt, 2)
    xin = spec.transpose(1, 2).reshape(b, nt, nf * s * 2)
    return spec, xin


def band_split(xin: torch.Tensor, sd: dict, cfg) -> torch.Tensor:
    """Per band: RMSNorm(din) then Linear(din -> dim); stacked on dim -2 (model.py:147-155).

    xin (b, T, 4F) -> X (b, T, n_bands, dim).
    """
    parts = xin.split(cfg.band_dims, dim=-1)
    outs = []
    for k, part in enumerate(parts):
        p = f"band_split.to_features.{k}."
        h = rmsnorm(part, sd[p + "0.gamma"])
        outs.append(F.linear(h, sd[p + "1.weight"], sd[p + "1.bias"]))
    return torch.stack(outs, dim=-2)


def axial_block(x: torch.Tensor, sd: dict, cfg, i: int) -> torch.Tensor:
    """One time transformer over frames, then one freq transformer over bands (model.py:262-268).

    x (b, T, nb, d) -> (b, T, nb, d).
    """
    b, nt, nb, d = x.shape
    x = x.transpose(1, 2).reshape(b * nb, nt, d)
    x = transformer(x, sd, f"layers.{i}.0.", cfg.heads, cfg.dim_head)
    x = x.view(b, nb, nt, d).transpose(1, 2).reshape(b * nt, nb, d)
    x = transformer(x, sd, f"layers.{i}.1.", cfg.heads, cfg.dim_head)
    return x.view(b, nt, nb, d)


def mask_estimator(x: torch.Tensor, sd: dict, cfg) -> torch.Tensor:
    """Per band: Linear -> Tanh -> Linear -> GLU, concatenated over bands (model.py:158-178).

    x (b, T, nb, d), already final-normed -> mask (b, T, 4F).
    """
    outs = []
    for k, band in enumerate(x.unbind(dim=-2)):
        p = f"mask_estimators.0.to_freqs.{k}.0."
        h = torch.tanh(F.linear(band, sd[p + "0.weight"], sd[p + "0.bias"]))
        o = F.linear(h, sd[p + "2.weight"], sd[p + "2.bias"])
        outs.append(F.glu(o, dim=-1))
    return torch.cat(outs, dim=-1)


def istft_apply(spec: torch.Tensor, mask: torch.Tensor, cfg) -> torch.Tensor:
    """Complex multiply by the mask, then iSTFT with the same window (model.py:271-277).

    spec (b, 2F, T, 2), mask (b, T, 4F) -> audio (b, 2, hop * (T - 1)).
    """
    b, nfs, nt, _ = spec.shape
    nf, s = nfs // 2, 2
    m = mask.view(b, 1, nt, nf * s, 2).permute(0, 1, 3, 2, 4)
    out = torch.view_as_complex(spec.unsqueeze(1).contiguous()) * torch.view_as_complex(m.contiguous())
    out = out.view(b, 1, nf, s, nt).permute(0, 1, 3, 2, 4).reshape(b * s, nf, nt)
    window = torch.hann_window(cfg.stft_win_length)
    audio = torch.istft(
        out,
        n_fft=cfg.stft_n_fft,
        hop_length=cfg.stft_hop_length,
        win_length=cfg.stft_win_length,
        normalized=False,
        window=window,
        return_complex=False,
    )
    return audio.view(b, s, -1)


@torch.inference_mode()
def forward(audio: torch.Tensor, sd: dict, cfg, stages: dict | None = None) -> torch.Tensor:
    """Full fp32 forward (model.py:247-278). audio (b, 2, L) -> (b, 2, hop * (L // hop)).

    If ``stages`` is a dict it receives the intermediate tensors: ``xin``, ``X0`` (after band split),
    ``X{i}`` (after axial block i), ``Xn`` (final-normed), ``mask``.
    """
    audio = audio.float()
    spec, xin = stft(audio, cfg)
    x = band_split(xin, sd, cfg)
    if stages is not None:
        stages["xin"] = xin
        stages["X0"] = x
    for i in range(cfg.depth):
        x = axial_block(x, sd, cfg, i)
        if stages is not None:
            stages[f"X{i + 1}"] = x
    x = rmsnorm(x, sd["final_norm.gamma"])
    mask = mask_estimator(x, sd, cfg)
    if stages is not None:
        stages["Xn"] = x
        stages["mask"] = mask
    return istft_apply(spec, mask, cfg)
