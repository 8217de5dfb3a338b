"""Protocol invariants of the attention kernel's key/value ring, checked on the host.

An mbarrier parity wait cannot tell phase u from phase u - 2, so every thread that waits on a stage
must wait on each of that stage's phases in order. The attention producer (`attention.cuh`) loads the
key/value tiles of item i into stages kvc % kAttnKvStages, kvc = loads issued so far; in frequency mode
there is one load per query tile and item (tile A, then tile B) and each tile's MMA issuer waits only on
its own loads, in time mode both tiles wait on every load. This test replays those schedules with the
stage count compiled into the kernel."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parents[1] / "turbo_roformer_b200" / "csrc" / "attention.cuh"


def kv_stages() -> int:
    m = re.search(r"constexpr int kAttnKvStages = (\d+);", HEADER.read_text())
    assert m, "kAttnKvStages not found"
    return int(m.group(1))


def waits_in_order(stages: int, loads_per_item: int, tiles_of_load, items: int = 64) -> bool:
    """True when every tile sees every phase of each stage it waits on, in order."""
    seen = {}  # (tile, stage) -> last use index waited on
    kvc = 0
    for _ in range(items):
        for j in range(loads_per_item):
            st, use = kvc % stages, kvc // stages
            for tile in tiles_of_load(j):
                last = seen.get((tile, st), -1)
                if use != last + 1:
                    return False
                seen[(tile, st)] = use
            kvc += 1
    return True


def test_frequency_mode_tiles_own_their_stages():
    s = kv_stages()
    assert waits_in_order(s, 2, lambda j: (j,))  # load j of an item belongs to tile j


def test_time_mode_both_tiles_wait_on_every_load():
    s = kv_stages()
    assert waits_in_order(s, 14, lambda j: (0, 1))  # T = 1700: 14 key tiles per item


@pytest.mark.parametrize("stages", [3, 5])
def test_odd_stage_counts_would_break_frequency_mode(stages):
    # the schedule the kernel used before the stage count became even
    assert not waits_in_order(stages, 2, lambda j: (j,))
