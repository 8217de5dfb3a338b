"""libtrcuda.so builds for sm_100a, loads without a GPU, and exports every symbol of include/trcuda.h."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from turbo_roformer_b200 import _build, _lib

from .conftest import REPO


def declared_symbols() -> list[str]:
    with open(os.path.join(REPO, "include", "trcuda.h")) as f:
        src = f.read()
    return sorted(set(re.findall(r"\b(trc_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("trc_create", "trc_set_param", "trc_prepare", "trc_forward", "trc_ola", "trc_destroy",
              "trc_last_error", "trc_attention", "trc_qkv_rope_gemm", "trc_gemm_res_norm", "trc_gemm_gelu",
              "trc_add_rmsnorm", "trc_stft", "trc_band_split", "trc_mask", "trc_istft", "trc_check",
              "trc_output_length"):
        assert s in syms, s


def test_library_builds_and_exports_every_declared_symbol():
    path = _build.build()
    lib = ctypes.CDLL(path)  # loading needs no GPU
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in include/trcuda.h but not exported"
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_loader_binds_signatures_and_reports_errors_without_gpu():
    lib = _lib.load()
    assert lib.trc_last_error() is not None
    # no device needed for argument validation
    h = ctypes.c_void_p()
    rc = lib.trc_create(None, 0, ctypes.byref(h))
    assert rc == -1
    assert b"null" in lib.trc_last_error()
    with pytest.raises(_lib.TRCError):
        _lib.check(rc)


def test_ola_rejects_bad_arguments_on_host():
    lib = _lib.load()
    starts = (ctypes.c_int64 * 2)(10, 5)  # not increasing
    rc = lib.trc_ola(ctypes.c_void_p(1), 100, starts, 2, 100, 1000, ctypes.c_void_p(1), None)
    assert rc == -1 and b"increasing" in lib.trc_last_error()


def test_built_for_sm100a_only():
    assert _build.ARCH_FLAGS == ("-gencode", "arch=compute_100a,code=sm_100a")
