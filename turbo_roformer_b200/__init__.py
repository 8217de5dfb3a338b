"""Blackwell (sm_100a) CUDA backend for the BS-RoFormer forward of turbo-roformer.

Public surface (mirrors the reference package): ``Separator`` (backend="cuda"; ``submit`` for queued
songs, ``stream`` for live input), ``CudaBSRoformer`` (the FastBSRoformer-compatible forward), the
chunking helpers, and the device channel fold / resampler (``remix_device``, ``resample_device``).
"""

from .chunking import chunk_starts, hamming, overlap_add, step_for
from .config import RESURRECTION, TINY, ModelConfig

__all__ = ["Separator", "SeparationJob", "SeparationStream", "CudaBSRoformer", "ModelConfig", "RESURRECTION", "TINY",
           "chunk_starts", "hamming", "overlap_add", "step_for", "remix_device", "resample_device"]


def __getattr__(name):
    if name in ("Separator", "SeparationJob", "SeparationStream"):
        from . import separator

        return getattr(separator, name)
    if name in ("remix_device", "resample_device"):
        from . import resample

        return getattr(resample, name)
    if name == "CudaBSRoformer":
        from .backend import CudaBSRoformer

        return CudaBSRoformer
    raise AttributeError(name)
