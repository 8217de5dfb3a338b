"""Architecture description of the BS-RoFormer checkpoints this backend runs.

The parameter tree mirrors the upstream BS-RoFormer ``state_dict`` keys exactly
(``turbo_roformer/model.py:114-278`` in LoggeL/turbo-roformer), so a checkpoint
that loads into the reference ``BSRoformer`` with ``strict=True`` loads here.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

# lucidrains' band layout (turbo_roformer/model.py:25): 62 bands over 1025 bins.
DEFAULT_FREQS_PER_BANDS: tuple[int, ...] = (2,) * 24 + (4,) * 12 + (12,) * 8 + (24,) * 8 + (48,) * 8 + (128, 129)


@dataclass(frozen=True)
class ModelConfig:
    """Hyper-parameters of one single-stem stereo BS-RoFormer.

    Mirrors the ``model:`` section of the reference configs (turbo_roformer/registry.py:49-69).
    Only what changes the inference math is kept.
    """

    dim: int = 256
    depth: int = 12
    heads: int = 8
    dim_head: int = 64
    ff_mult: int = 4
    freqs_per_bands: tuple[int, ...] = DEFAULT_FREQS_PER_BANDS
    stft_n_fft: int = 2048
    stft_hop_length: int = 441
    stft_win_length: int = 2048
    mlp_expansion_factor: int = 4
    mask_estimator_depth: int = 2
    audio_channels: int = 2
    num_stems: int = 1
    time_transformer_depth: int = 1
    freq_transformer_depth: int = 1
    dim_t: int = 1700  # inference chunk in frames: chunk = hop * (dim_t - 1) (registry.py:84-85)
    extra: dict = field(default_factory=dict, compare=False)

    @property
    def n_bands(self) -> int:
        return len(self.freqs_per_bands)

    @property
    def n_freqs(self) -> int:
        return self.stft_n_fft // 2 + 1

    @property
    def band_dims(self) -> tuple[int, ...]:
        """Per-band input width: freqs x stereo x (re, im) (model.py:238)."""
        return tuple(2 * f * self.audio_channels for f in self.freqs_per_bands)

    @property
    def ff_inner(self) -> int:
        return self.dim * self.ff_mult

    @property
    def mask_hidden(self) -> int:
        return self.dim * self.mlp_expansion_factor

    @property
    def chunk(self) -> int:
        return self.stft_hop_length * (self.dim_t - 1)

    def validate_for_cuda(self) -> None:
        """The CUDA backend supports what the reference's fast CPU path supports (fast.py:106-134): besides
        256, any width that is a multiple of 64 up to 1024 (there the reference drops its fused kernels,
        fast.py:121-122; here the 256-only fused epilogues are replaced by fp32 residual-branch GEMMs and
        row norms)."""
        if self.num_stems != 1 or self.audio_channels != 2:
            raise NotImplementedError("only single-stem stereo BS-RoFormer models are supported")
        if (self.heads, self.dim_head) != (8, 64):
            raise NotImplementedError(f"only heads=8, dim_head=64 is supported (got {self.heads}, {self.dim_head})")
        if self.dim % 64 or not 128 <= self.dim <= 1024:
            raise NotImplementedError(f"dim must be a multiple of 64 in [128, 1024] (got {self.dim})")
        if self.time_transformer_depth != 1 or self.freq_transformer_depth != 1:
            raise NotImplementedError("only time/freq transformer depth 1 is supported")
        if self.mask_estimator_depth != 2:
            raise NotImplementedError("only mask_estimator_depth=2 is supported")
        if sum(self.freqs_per_bands) != self.n_freqs:
            raise ValueError(f"freqs_per_bands must sum to {self.n_freqs}")
        n = self.stft_n_fft
        if n & (n - 1) or not (256 <= n <= 4096):
            raise NotImplementedError("stft_n_fft must be a power of two in [256, 4096]")
        if self.stft_win_length != n:
            raise NotImplementedError("stft_win_length must equal stft_n_fft")
        if self.ff_inner % 64 or self.mask_hidden % 64:
            raise NotImplementedError("ff and mask hidden widths must be multiples of 64")
        if self.n_bands > 64:
            raise NotImplementedError("at most 64 bands are supported")
        if max(self.band_dims) > 1024 or max(self.band_dims) * 2 > 2048:
            raise NotImplementedError("band widths above 1024 are not supported")


# "BS Roformer | Instrumental Resurrection by unwa" (turbo_roformer/registry.py:49-69)
RESURRECTION = ModelConfig()

# Small but structurally complete model used by the reference's tests (tests/conftest.py:14-33):
# 2 axial blocks, n_fft 512 (257 bins in 29 bands), hop 128, 128-frame chunks.
TINY = ModelConfig(
    depth=2,
    freqs_per_bands=(4,) * 16 + (8,) * 8 + (16,) * 4 + (65,),
    stft_n_fft=512,
    stft_hop_length=128,
    stft_win_length=512,
    mlp_expansion_factor=2,
    dim_t=128,
)


def param_shapes(cfg: ModelConfig) -> "OrderedDict[str, tuple[int, ...]]":
    """Upstream ``state_dict`` keys and shapes, in module registration order (model.py:181-245)."""
    d, H, Dh = cfg.dim, cfg.heads, cfg.dim_head
    inner = H * Dh
    out: OrderedDict[str, tuple[int, ...]] = OrderedDict()
    for i in range(cfg.depth):
        for j in range(2):  # 0 = time transformer, 1 = freq transformer
            p = f"layers.{i}.{j}.layers.0."
            out[p + "0.rotary_embed.freqs"] = (Dh // 2,)
            out[p + "0.norm.gamma"] = (d,)
            out[p + "0.to_qkv.weight"] = (3 * inner, d)
            out[p + "0.to_gates.weight"] = (H, d)
            out[p + "0.to_gates.bias"] = (H,)
            out[p + "0.to_out.0.weight"] = (d, inner)
            out[p + "1.net.0.gamma"] = (d,)
            out[p + "1.net.1.weight"] = (cfg.ff_inner, d)
            out[p + "1.net.1.bias"] = (cfg.ff_inner,)
            out[p + "1.net.4.weight"] = (d, cfg.ff_inner)
            out[p + "1.net.4.bias"] = (d,)
    out["final_norm.gamma"] = (d,)
    for k, din in enumerate(cfg.band_dims):
        out[f"band_split.to_features.{k}.0.gamma"] = (din,)
        out[f"band_split.to_features.{k}.1.weight"] = (d, din)
        out[f"band_split.to_features.{k}.1.bias"] = (d,)
    for k, din in enumerate(cfg.band_dims):
        p = f"mask_estimators.0.to_freqs.{k}.0."
        out[p + "0.weight"] = (cfg.mask_hidden, d)
        out[p + "0.bias"] = (cfg.mask_hidden,)
        out[p + "2.weight"] = (2 * din, cfg.mask_hidden)
        out[p + "2.bias"] = (2 * din,)
    return out


def infer_config(state_dict, hop: int, dim_t: int) -> ModelConfig:
    """Recover the architecture from an upstream ``state_dict`` plus the STFT hop and chunk frames.

    Hop and chunk length are not stored in checkpoints; the caller passes them like
    ``Separator.from_module(net, hop, dim_t)`` (turbo_roformer/separator.py:160-179).
    """
    sd = state_dict
    dim = int(sd["final_norm.gamma"].shape[0])
    depth = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("layers."))
    tdepth = 1 + max(int(k.split(".")[4]) for k in sd if k.startswith("layers.0.0.layers."))
    fdepth = 1 + max(int(k.split(".")[4]) for k in sd if k.startswith("layers.0.1.layers."))
    n_bands = 1 + max(int(k.split(".")[2]) for k in sd if k.startswith("band_split.to_features."))
    dims = [int(sd[f"band_split.to_features.{k}.0.gamma"].shape[0]) for k in range(n_bands)]
    if any(x % 4 for x in dims):
        raise NotImplementedError("only stereo models (band widths multiple of 4) are supported")
    freqs = tuple(x // 4 for x in dims)
    n_fft = 2 * (sum(freqs) - 1)
    qkv = sd["layers.0.0.layers.0.0.to_qkv.weight"]
    n_rot = int(sd["layers.0.0.layers.0.0.rotary_embed.freqs"].shape[0])
    dim_head = 2 * n_rot
    heads = int(qkv.shape[0]) // (3 * dim_head)
    ff_inner = int(sd["layers.0.0.layers.0.1.net.1.weight"].shape[0])
    mask_hidden = int(sd["mask_estimators.0.to_freqs.0.0.0.weight"].shape[0])
    mdepth = sum(1 for k in sd if k.startswith("mask_estimators.0.to_freqs.0.0.") and k.endswith(".weight"))
    n_stems = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("mask_estimators."))
    return ModelConfig(
        dim=dim,
        depth=depth,
        heads=heads,
        dim_head=dim_head,
        ff_mult=ff_inner // dim,
        freqs_per_bands=freqs,
        stft_n_fft=n_fft,
        stft_hop_length=int(hop),
        stft_win_length=n_fft,
        mlp_expansion_factor=mask_hidden // dim,
        mask_estimator_depth=mdepth,
        num_stems=n_stems,
        time_transformer_depth=tdepth,
        freq_transformer_depth=fdepth,
        dim_t=int(dim_t),
    )
