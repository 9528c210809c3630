"""Host-side step metadata: what the scheduler hands the kernels.

The reference passes one sequence's block table as a Python list and its
start position as an int per ``forward_step`` call (engine/runner.py:65-79,
engine/model.py:149). A batched step instead carries, for B sequences,
  cu_q        int32 (B+1,)  cumulative chunk lengths (row offsets into q)
  start_pos   int32 (B,)    absolute position of each chunk's first token
  block_tables int32 (B, max_blocks)  padded with -1
all in one contiguous int32 buffer so a single host->device copy moves it.
The validation here mirrors the reference's failure mode: a block table too
short for its context raises IndexError (engine/paged_attention.py:77, 95).
"""

from __future__ import annotations

import itertools

import numpy as np


def validate_tables(q_lens, start_pos, block_tables, block_size: int) -> list[int]:
    B = len(q_lens)
    if not (len(start_pos) == B == len(block_tables)):
        raise ValueError("q_lens, start_pos and block_tables need one entry per sequence")
    if B == 0:
        raise ValueError("empty batch")
    ctx = []
    for b in range(B):
        if q_lens[b] <= 0:
            raise ValueError(f"sequence {b}: empty chunk")
        if start_pos[b] < 0:
            raise ValueError(f"sequence {b}: negative start position")
        c = int(start_pos[b]) + int(q_lens[b])
        need = (c + block_size - 1) // block_size
        if len(block_tables[b]) < need:
            raise IndexError(f"sequence {b}: block_table has {len(block_tables[b])} entries, context {c} "
                             f"needs {need}")
        ctx.append(c)
    return ctx


def pack_metadata(q_lens, start_pos, block_tables, block_size: int, num_blocks: int | None = None,
                  max_blocks: int | None = None) -> tuple[np.ndarray, int, int, list[int]]:
    """-> (int32 buffer [cu_q | start_pos | tables], B, max_blocks, ctx_lens).
    Block ids outside [0, num_blocks) raise IndexError (the kernels would
    skip them and set the device status word)."""
    ctx = validate_tables(q_lens, start_pos, block_tables, block_size)
    B = len(q_lens)
    lens = [len(t) for t in block_tables]
    mb = max_blocks or max(1, max(lens))
    # one flat conversion of all tables and vectorised checks: this runs on
    # the host between steps, so its cost is part of the end-to-end step
    n = np.minimum(np.asarray(lens, np.int64), mb)
    short = np.nonzero(n < (np.asarray(ctx, np.int64) + block_size - 1) // block_size)[0]
    if short.size:
        b = int(short[0])
        raise IndexError(f"sequence {b}: context {ctx[b]} exceeds max_blocks {mb}")
    total = int(n.sum())
    flat = np.fromiter(itertools.chain.from_iterable(t[:mb] if len(t) > mb else t for t in block_tables),
                       dtype=np.int64, count=total)
    if num_blocks is not None and total:
        bad = (flat < 0) | (flat >= num_blocks)
        if bad.any():
            b = int(np.searchsorted(np.cumsum(n), int(np.argmax(bad)), side="right"))
            raise IndexError(f"sequence {b}: block id outside the pool of {num_blocks} blocks")
    tab = np.full((B, mb), -1, dtype=np.int32)
    if total:
        starts = np.cumsum(n) - n
        tab[np.repeat(np.arange(B), n), np.arange(total) - np.repeat(starts, n)] = flat
    cu = np.zeros(B + 1, dtype=np.int32)
    cu[1:] = np.cumsum(np.asarray(q_lens, dtype=np.int64))
    buf = np.concatenate([cu, np.asarray(start_pos, np.int32), tab.reshape(-1)])
    return buf, B, mb, ctx


def attention_runs(q_lens, group: int, rows_per_decode_tile: int = 16) -> list[tuple[int, int, bool]]:
    """Split a batch into maximal runs of consecutive sequences that use the
    same attention kernel: decode (q_len * group <= 16 rows, split-context
    kernel) or prefill (row-tiled kernel). -> [(begin, end, is_decode)]."""
    kinds = [q * group <= rows_per_decode_tile for q in q_lens]
    runs = []
    s = 0
    for i in range(1, len(kinds) + 1):
        if i == len(kinds) or kinds[i] != kinds[s]:
            runs.append((s, i, kinds[s]))
            s = i
    return runs


def slot_mapping(q_lens, start_pos, block_tables, block_size: int) -> tuple[np.ndarray, np.ndarray]:
    """Host restatement of ps_build_slot_mapping for checking: positions and
    slots (block_table[pos // bs] * bs + pos % bs, engine/paged_attention.py:74-77)."""
    pos, slots = [], []
    for q, s, t in zip(q_lens, start_pos, block_tables):
        for i in range(q):
            p = s + i
            pos.append(p)
            slots.append(t[p // block_size] * block_size + p % block_size)
    return np.asarray(pos, np.int32), np.asarray(slots, np.int32)
