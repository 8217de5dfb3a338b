"""``CudaBSRoformer``: the B200 forward behind the reference's ``FastBSRoformer`` contract.

``CudaBSRoformer(model_or_state_dict, ...)(raw_audio)`` maps (1, 2, samples) float32 to
(1, 2, hop * (samples // hop)) exactly like ``FastBSRoformer.forward`` (turbo_roformer/fast.py:363-394),
and additionally accepts a batch (B, 2, samples) of equal-length chunks. Input may live on the CPU or on
the handle's GPU; the output is returned on the input's device. All numerics run in libtrcuda.so
(sm_100a kernels); there is no CPU fallback: without the library, construction raises
``KernelUnavailable``.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from .config import ModelConfig, infer_config

PRECISIONS = {"fp16": _lib.TRC_PREC_FP16, "bf16": _lib.TRC_PREC_BF16}


def _state_dict_of(model) -> dict:
    if isinstance(model, dict):
        return model
    if hasattr(model, "state_dict"):
        return model.state_dict()
    raise TypeError("expected a BS-RoFormer module or an upstream state_dict")


class CudaBSRoformer:
    """One model replica on one GPU. One forward at a time per instance (the work buffers are shared)."""

    def __init__(
        self,
        model,
        cfg: ModelConfig | None = None,
        device: int | torch.device | None = None,
        precision: str = "fp16",
        hop: int | None = None,
        dim_t: int | None = None,
    ):
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {tuple(PRECISIONS)} for the cuda backend")
        sd = _state_dict_of(model)
        if cfg is None:
            if hop is None:
                hop = getattr(model, "stft_kwargs", {}).get("hop_length")
            if hop is None:
                raise ValueError("pass cfg=ModelConfig(...) or hop= (the STFT hop is not stored in checkpoints)")
            cfg = infer_config(sd, hop=int(hop), dim_t=int(dim_t or 801))
        cfg.validate_for_cuda()
        if not torch.cuda.is_available():
            raise _lib.KernelUnavailable("the cuda backend needs a CUDA device (none visible)")
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", torch.device(device).index if not isinstance(device, int) else device)
        self.cfg = cfg
        self.precision = precision
        self.hop = cfg.stft_hop_length
        self.lib = _lib.load()
        self._lock = threading.Lock()
        freqs = (ctypes.c_int * cfg.n_bands)(*cfg.freqs_per_bands)
        c = _lib.TRCConfig(
            dim=cfg.dim,
            depth=cfg.depth,
            heads=cfg.heads,
            dim_head=cfg.dim_head,
            ff_mult=cfg.ff_mult,
            n_bands=cfg.n_bands,
            freqs_per_band=freqs,
            n_fft=cfg.stft_n_fft,
            hop=cfg.stft_hop_length,
            win_length=cfg.stft_win_length,
            mlp_expansion_factor=cfg.mlp_expansion_factor,
            precision=PRECISIONS[precision],
        )
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.trc_create(ctypes.byref(c), self.device.index, ctypes.byref(h)))
        self._h = h
        try:
            for name, t in sd.items():
                if name.endswith("rotary_embed.freqs") or name.startswith(("layers.", "final_norm.", "band_split.", "mask_estimators.")):
                    a = t.detach().to("cpu", torch.float32).contiguous()
                    _lib.check(self.lib.trc_set_param(h, name.encode(), ctypes.c_void_p(a.data_ptr()), a.numel()))
            with torch.cuda.device(self.device):
                _lib.check(self.lib.trc_prepare(h))
        except Exception:
            self.close()
            raise

    # ------------------------------------------------------------------ lifetime
    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self.lib.trc_destroy(h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise RuntimeError("CudaBSRoformer is closed")
        return self._h

    def stream_ptr(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def output_length(self, samples: int) -> int:
        return self.hop * (samples // self.hop)

    def check(self) -> None:
        """Synchronise the current stream and raise if a kernel reported a device-side error."""
        _lib.check(self.lib.trc_check(self.handle, ctypes.c_void_p(self.stream_ptr())))

    def error_async(self, host_word: torch.Tensor) -> None:
        """Queue a copy of the device error word into ``host_word`` (pinned int32, 1 element) on the
        current stream and clear the device word; read it after the stream has passed this point."""
        if host_word.dtype != torch.int32 or host_word.device.type != "cpu" or not host_word.is_pinned():
            raise ValueError("host_word must be a pinned int32 CPU tensor")
        _lib.check(self.lib.trc_error_async(self.handle, ctypes.c_void_p(host_word.data_ptr()),
                                            ctypes.c_void_p(self.stream_ptr())))

    # ------------------------------------------------------------------ forward
    def forward_device(self, audio: torch.Tensor, out: torch.Tensor | None = None, check: bool = True) -> torch.Tensor:
        """audio (B, 2, L) float32 on this GPU -> (B, 2, hop * (L // hop)) on this GPU (current stream)."""
        if audio.ndim != 3 or audio.shape[1] != 2:
            raise ValueError(f"expected (batch, 2, samples), got {tuple(audio.shape)}")
        if audio.device != self.device or audio.dtype != torch.float32:
            raise ValueError("forward_device expects float32 input on the model's device")
        audio = audio.contiguous()
        B, _, L = audio.shape
        if L <= self.cfg.stft_n_fft // 2:
            raise ValueError(f"need more than n_fft/2 = {self.cfg.stft_n_fft // 2} samples, got {L}")
        lo = self.output_length(L)
        if out is None:
            out = torch.empty(B, 2, lo, device=self.device, dtype=torch.float32)
        elif out.shape != (B, 2, lo) or not out.is_contiguous() or out.device != self.device:
            raise ValueError("bad output buffer")
        with self._lock, torch.cuda.device(self.device):
            rc = self.lib.trc_forward(
                self.handle,
                ctypes.c_void_p(audio.data_ptr()),
                B,
                L,
                ctypes.c_void_p(out.data_ptr()),
                ctypes.c_void_p(self.stream_ptr()),
            )
            _lib.check(rc)
            if check:
                self.check()
        return out

    def transformer_device(self, X: torch.Tensor, batch: int, T: int, check: bool = True) -> torch.Tensor:
        """The 2*depth transformers alone (``FastBSRoformer._transformer_cpp``, fast.py:269-341) on the fp32
        residual stream X (batch * T * n_bands, dim) on this GPU, updated in place and returned."""
        if X.shape != (batch * T * self.cfg.n_bands, self.cfg.dim) or X.dtype != torch.float32:
            raise ValueError(f"expected X of shape ({batch * T * self.cfg.n_bands}, {self.cfg.dim}) float32")
        if X.device != self.device or not X.is_contiguous():
            raise ValueError("X must be a contiguous tensor on the model's device")
        with self._lock, torch.cuda.device(self.device):
            _lib.check(self.lib.trc_transformer(self.handle, ctypes.c_void_p(X.data_ptr()), batch, T,
                                                ctypes.c_void_p(self.stream_ptr())))
            if check:
                self.check()
        return X

    @torch.inference_mode()
    def forward(self, raw_audio: torch.Tensor) -> torch.Tensor:
        """(B, 2, samples) float32 -> (B, 2, hop * (samples // hop)), on the input's device."""
        if raw_audio.ndim != 3 or raw_audio.shape[1] != 2:
            raise ValueError(f"expected (1, 2, samples), got {tuple(raw_audio.shape)}")
        src = raw_audio.device
        x = raw_audio.to(self.device, torch.float32, non_blocking=False)
        y = self.forward_device(x)
        return y if src == self.device else y.to(src)

    __call__ = forward

    def release_buffers(self) -> None:
        """Work buffers are owned by the library handle and reused; kept for API parity with FastBSRoformer."""
        return None
