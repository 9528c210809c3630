"""Host logic of prefix sharing (pageserve_b200/prefix.py), on CPU: a forked
sequence shares every full block of its parent's table and gets a new block,
to be filled by copy-on-write, for a partly filled last block — the device
side of engine/prefix_cache.py:35-82's shared physical blocks."""

import pytest

from pageserve_b200.prefix import fork_block_table


def _alloc(start):
    it = iter(range(start, 1000))
    return lambda: next(it)


def test_fork_shares_full_blocks_and_copies_the_partial_one():
    table, copies = fork_block_table([7, 3, 9, 4, 11], 14, 4, _alloc(50))
    assert table == [7, 3, 9, 50] and copies == [(4, 50)]


def test_fork_at_a_block_boundary_copies_nothing():
    table, copies = fork_block_table([7, 3, 9], 12, 4, _alloc(50))
    assert table == [7, 3, 9] and copies == []
    table, copies = fork_block_table([7, 3, 9], 0, 4, _alloc(50))
    assert table == [] and copies == []


def test_fork_of_a_short_table_raises_index_error():
    with pytest.raises(IndexError):
        fork_block_table([7, 3], 9, 4, _alloc(50))
