"""The multi-GPU song path (`separate_song_from_host`) on one GPU as a one-rank NCCL group: span copy,
peak reduction, the shard's forwards, the gather and the rank-0 overlap-add on the side stream must
give exactly `Separator.separate`'s result. (Two or more ranks are covered on CPU by the gloo tests and
measured by `bench.py --gpus N`.)"""

from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist

from turbo_roformer_b200 import synthetic as S

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_song_from_host_on_one_rank_equals_separate(tiny_sd, tiny_cfg, cuda_device):
    from turbo_roformer_b200.distributed import separate_song_from_host
    from turbo_roformer_b200.separator import Separator

    sep = Separator.from_module(tiny_sd, tiny_cfg.stft_hop_length, tiny_cfg.dim_t, batch=3)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
    try:
        for k, overlap in enumerate((2.0, 3.0)):
            mix = (S.chunk_audio(44100 * 3 + 123 * k, seed=90 + k) * 4.0).astype(np.float32)  # peak gain path
            ref = sep.separate(mix, overlap=overlap)
            out = torch.empty(2, mix.shape[1], dtype=torch.float32).pin_memory()
            for _ in range(2):  # queued twice without a host synchronisation in between
                separate_song_from_host(sep, torch.from_numpy(mix).pin_memory(), overlap, out=out)
            torch.cuda.synchronize()
            sep.net.check()
            np.testing.assert_array_equal(out.numpy(), ref)
    finally:
        dist.destroy_process_group()
