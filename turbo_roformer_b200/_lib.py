"""ctypes binding of libtrcuda.so (the C ABI in include/trcuda.h).

Mirrors the reference's kernel loader (turbo_roformer/_kernels.py:112-144): ``load()`` returns the
library or raises ``KernelUnavailable``; there is no silent fallback. A failing call raises
``TRCError`` with the library's message.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import _build

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

TRC_PREC_FP16 = 0
TRC_PREC_BF16 = 1
TRC_E_DEVICE = -3  # a kernel reported a device-side error (include/trcuda.h)

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_f = ctypes.c_float
c_vp = ctypes.c_void_p
c_char_p = ctypes.c_char_p


class KernelUnavailable(RuntimeError):
    """The CUDA library could not be built or loaded."""


class TRCError(RuntimeError):
    """A libtrcuda call returned an error code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libtrcuda error {code}: {msg}")
        self.code = code


class TRCConfig(ctypes.Structure):
    _fields_ = [
        ("dim", c_int),
        ("depth", c_int),
        ("heads", c_int),
        ("dim_head", c_int),
        ("ff_mult", c_int),
        ("n_bands", c_int),
        ("freqs_per_band", ctypes.POINTER(c_int)),
        ("n_fft", c_int),
        ("hop", c_int),
        ("win_length", c_int),
        ("mlp_expansion_factor", c_int),
        ("precision", c_int),
    ]


# name -> (restype, argtypes): every symbol declared in include/trcuda.h
SIGNATURES = {
    "trc_create": (c_int, [ctypes.POINTER(TRCConfig), c_int, ctypes.POINTER(c_vp)]),
    "trc_set_param": (c_int, [c_vp, c_char_p, c_vp, c_i64]),
    "trc_prepare": (c_int, [c_vp]),
    "trc_destroy": (None, [c_vp]),
    "trc_forward": (c_int, [c_vp, c_vp, c_int, c_i64, c_vp, c_vp]),
    "trc_output_length": (c_i64, [c_vp, c_i64]),
    "trc_transformer": (c_int, [c_vp, c_vp, c_int, c_int, c_vp]),
    "trc_check": (c_int, [c_vp, c_vp]),
    "trc_error_async": (c_int, [c_vp, c_vp, c_vp]),
    "trc_selftest_wait_timeout": (c_int, [c_vp, c_vp]),
    "trc_ola": (c_int, [c_vp, c_i64, c_vp, c_int, c_i64, c_i64, c_vp, c_vp]),
    "trc_last_error": (c_char_p, []),
    "trc_remix": (c_int, [c_vp, c_int, c_i64, c_vp, c_vp, c_vp]),
    "trc_resample": (c_int, [c_vp, c_int, c_i64, c_int, c_int, c_i64, c_vp, c_int, c_i64, c_vp, c_vp]),
    "trc_ola_noalloc": (c_int, [c_vp, c_i64, c_vp, c_int, c_i64, c_i64, c_vp, c_vp]),
    "trc_profile": (c_int, [c_vp, c_int]),
    "trc_profile_read": (c_int, [c_vp, c_char_p, c_int]),
    "trc_launch_count": (ctypes.c_longlong, []),
    "trc_add_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_f, c_vp]),
    "trc_qkv_rope_gemm": (c_int, [c_vp, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "trc_attention": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_vp]),
    "trc_gemm_res_norm": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "trc_gemm_gelu": (c_int, [c_vp, c_int, c_vp, c_vp, c_i64, c_vp]),
    "trc_ffn_res_norm": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "trc_rope_pack": (c_int, [c_vp, c_int, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "trc_gate_merge": (c_int, [c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_vp]),
    "trc_stft": (c_int, [c_vp, c_vp, c_int, c_i64, c_vp, c_vp]),
    "trc_band_split": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    "trc_mask": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    "trc_istft": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
}


def library_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) libtrcuda.so; raises KernelUnavailable on failure."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if os.environ.get("TURBO_ROFORMER_DISABLE_KERNELS"):
            raise KernelUnavailable("disabled by TURBO_ROFORMER_DISABLE_KERNELS")
        path = library_path()
        try:
            if build_if_missing:
                path = _build.build()
            elif not os.path.exists(path):
                raise KernelUnavailable(f"{path} is missing; run python -m turbo_roformer_b200._build")
            lib = ctypes.CDLL(path)
        except KernelUnavailable:
            raise
        except Exception as e:  # nvcc missing, compile error, dlopen failure
            raise KernelUnavailable(str(e)) from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def is_loaded() -> bool:
    return _lib is not None


def check(rc: int) -> None:
    if rc != 0:
        msg = load().trc_last_error()
        raise TRCError(rc, msg.decode() if msg else "unknown error")
