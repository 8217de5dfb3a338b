"""Blackwell (sm_100a) CUDA backend for the BS-RoFormer forward of turbo-roformer.

Public surface (mirrors the reference package): ``Separator`` (backend="cuda"), ``CudaBSRoformer``
(the FastBSRoformer-compatible forward), and the chunking helpers.
"""

from .chunking import chunk_starts, hamming, overlap_add, step_for
from .config import RESURRECTION, TINY, ModelConfig

__all__ = ["Separator", "CudaBSRoformer", "ModelConfig", "RESURRECTION", "TINY", "chunk_starts", "hamming",
           "overlap_add", "step_for"]


def __getattr__(name):
    if name == "Separator":
        from .separator import Separator

        return Separator
    if name == "CudaBSRoformer":
        from .backend import CudaBSRoformer

        return CudaBSRoformer
    raise AttributeError(name)
