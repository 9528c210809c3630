"""CUDA-graph buckets for the step (engine/cuda_graphs.py:13-26, 32-69).

The reference captures one decode graph per batch size (``DecodeGraph``) but
cannot replay it at a new position: its write_kv/gather_kv take Python ints
and lists. ``StepGraph`` keeps token ids, start positions and block tables in
device buffers refreshed by copies, so one graph serves every step of one
shape. ``StepGraphs`` picks the graph for each step:

* decode steps (every sequence feeds one token) run in the smallest captured
  batch bucket that holds them (``decode_buckets``, powers of two by
  default); the unused rows are pad sequences that decode token 0 at
  position 0 into ``pad_block``, a block of the pool the caller reserves for
  this (its contents are scratch), and their tokens are dropped;
* any other step (chunked prefill mixed with decodes) runs in a graph of its
  exact chunk lengths, captured on first use and kept in a bounded LRU.

Every graph is captured from the first step that needs it (the capture's
warm-up runs that step, writing the same KV it would write anyway).
"""

from __future__ import annotations

from collections import OrderedDict

import numpy as np

from .model import StepGraph


class StepGraphs:
    def __init__(self, model, max_blocks: int, max_ctx: int, pad_block: int,
                 decode_buckets=(1, 2, 4, 8, 16, 32, 64, 128, 256), max_mixed_graphs: int = 8):
        if not 0 <= pad_block < model.num_blocks:
            raise IndexError(f"pad_block {pad_block} outside the pool of {model.num_blocks}")
        self.m = model
        self.max_blocks = max_blocks
        self.max_ctx = max_ctx
        self.pad_block = pad_block
        self.decode_buckets = sorted(decode_buckets)
        self.max_mixed = max_mixed_graphs
        self.decode: dict[int, StepGraph] = {}
        self.mixed: OrderedDict[tuple, StepGraph] = OrderedDict()
        self.captures = 0

    def bucket(self, n: int) -> int | None:
        for b in self.decode_buckets:
            if b >= n:
                return b
        return None

    def _capture(self, q_lens, start_pos, tables, ids) -> StepGraph:
        self.captures += 1
        return StepGraph(self.m, list(q_lens), self.max_blocks, self.max_ctx, list(start_pos), tables, input_ids=ids)

    def run(self, input_ids, q_lens: list[int], start_pos: list[int], block_tables: list[list[int]]) -> np.ndarray:
        """One step through its graph: host inputs in, host next tokens (one
        per sequence, int32) out."""
        ids = np.asarray(input_ids, np.int64).reshape(-1)
        n = len(q_lens)
        if all(q == 1 for q in q_lens) and self.bucket(n) is not None:
            B = self.bucket(n)
            pad = B - n
            ids_p = np.concatenate([ids, np.zeros(pad, np.int64)])
            sp = list(start_pos) + [0] * pad
            tabs = [list(t) for t in block_tables] + [[self.pad_block]] * pad
            g = self.decode.get(B)
            if g is None:
                g = self.decode[B] = self._capture([1] * B, sp, tabs, ids_p)
            return g.run(ids_p, sp, tabs)[:n]
        key = tuple(int(q) for q in q_lens)
        g = self.mixed.get(key)
        if g is None:
            g = self._capture(key, start_pos, block_tables, ids)
            self.mixed[key] = g
            while len(self.mixed) > self.max_mixed:
                _, old = self.mixed.popitem(last=False)
                old.release()
        else:
            self.mixed.move_to_end(key)
        return g.run(ids, start_pos, block_tables)

    def logits(self, n: int, q_lens: list[int] | None = None):
        """The last step's logits rows of its n sequences (the graph's output
        buffer: valid until that graph's next replay)."""
        if q_lens is not None and not all(q == 1 for q in q_lens):
            return self.mixed[tuple(q_lens)].logits[:n]
        return self.decode[self.bucket(n)].logits[:n]

    def release(self) -> None:
        for g in list(self.decode.values()) + list(self.mixed.values()):
            g.release()
        self.decode.clear()
        self.mixed.clear()
