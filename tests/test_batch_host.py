"""Host-side step metadata (pageserve_b200/batch.py) on CPU."""

import numpy as np
import pytest

from oracle import ops
from pageserve_b200 import batch


def test_pack_metadata_layout():
    buf, B, mb, ctx = batch.pack_metadata([1, 3], [5, 0], [[7, 1], [2]], block_size=4, num_blocks=10)
    assert B == 2 and mb == 2 and ctx == [6, 3]
    # cu_q | start_pos | tables
    assert buf[:3].tolist() == [0, 1, 4]
    assert buf[3:5].tolist() == [5, 0]
    assert buf[5:].reshape(2, 2).tolist() == [[7, 1], [2, -1]]


def test_short_block_table_raises_index_error_like_reference():
    with pytest.raises(IndexError):
        batch.pack_metadata([1], [16], [[3]], block_size=16)
    with pytest.raises(IndexError):
        batch.pack_metadata([2], [0], [[11]], block_size=16, num_blocks=10)


def test_attention_runs():
    assert batch.attention_runs([1, 1, 512, 1], group=8) == [(0, 2, True), (2, 3, False), (3, 4, True)]
    assert batch.attention_runs([2, 3], group=8) == [(0, 1, True), (1, 2, False)]


def test_slot_mapping_matches_oracle_slots():
    rng = np.random.default_rng(0)
    tables = [list(rng.permutation(64)[:8]), list(rng.permutation(64)[:5])]
    pos, slots = batch.slot_mapping([3, 1], [10, 70], tables, 16)
    assert pos.tolist() == [10, 11, 12, 70]
    for p, s, t in zip(pos, slots, [tables[0]] * 3 + [tables[1]]):
        blk, off = ops.slot_of(t, 16, int(p))
        assert s == blk * 16 + off
