"""Prefix-cache-aware block sharing on the device-side KV layout.

The reference's prefix cache (engine/prefix_cache.py:35-82) lets sequences
that share a token prefix share physical KV blocks: its block tables simply
name the same block ids, with a reference count per block. The kernels here
read blocks in place through each sequence's table, so shared ids need
nothing from them. What sharing does need on the device is copy-on-write:
a sequence that continues from a shared block that is only partly filled
(a fork after a prompt that ends mid-block, e.g. several samples from one
prompt) must write its next tokens into a private copy of that block, or it
would overwrite the other sequences' rows.

* :func:`copy_blocks` copies whole blocks of every layer of both caches.
* :func:`fork_block_table` gives a forked sequence its table: every full
  block shared, the partial last block (if any) copied into a new block.
"""

from __future__ import annotations

from typing import Callable

import torch

from . import _lib


def copy_blocks(k_cache: torch.Tensor, v_cache: torch.Tensor, pairs) -> None:
    """For each (src, dst) block id pair, block dst of every layer of both
    caches ((L, NB, bs, Hkv, D), engine/model.py:143-147) becomes a copy of
    block src (on the current stream). Raises IndexError for ids outside the
    pool."""
    _lib.require_cuda(k_cache, v_cache)
    if k_cache.shape != v_cache.shape or k_cache.dtype != v_cache.dtype:
        raise ValueError("copy_blocks: K and V caches differ in shape or dtype")
    if k_cache.dim() == 4:  # one layer's (NB, bs, Hkv, D) cache
        k_cache, v_cache = k_cache.unsqueeze(0), v_cache.unsqueeze(0)
    L, NB, bs, hkv, d = k_cache.shape
    flat = [int(x) for p in pairs for x in p]
    if not flat:
        return
    if any(b < 0 or b >= NB for b in flat):
        raise IndexError(f"copy_blocks: block id outside the pool of {NB}")
    dev_pairs = torch.tensor(flat, dtype=torch.int32, device=k_cache.device)
    _lib.check(_lib.load().ps_copy_kv_blocks(k_cache.data_ptr(), v_cache.data_ptr(), dev_pairs.data_ptr(),
                                             len(flat) // 2, L, NB, bs, hkv, d, _lib.dtype_code(k_cache.dtype),
                                             _lib.stream_ptr(k_cache.device)), "copy_kv_blocks")


def fork_block_table(block_table: list[int], num_tokens: int, block_size: int,
                     allocate: Callable[[], int]) -> tuple[list[int], list[tuple[int, int]]]:
    """The table of a sequence forked from one holding ``num_tokens`` tokens
    in ``block_table``: the full blocks are shared (same ids), and a partly
    filled last block is replaced by a new block from ``allocate()``, to be
    filled by copy-on-write. Returns (new table, [(src, dst)] copies to make
    with :func:`copy_blocks` before the fork writes)."""
    full = num_tokens // block_size
    if (num_tokens + block_size - 1) // block_size > len(block_table):
        raise IndexError(f"block_table has {len(block_table)} entries for {num_tokens} tokens")
    table = list(block_table[:full])
    copies = []
    if num_tokens % block_size:
        new = int(allocate())
        copies.append((int(block_table[full]), new))
        table.append(new)
    return table, copies


def fork(model, block_table: list[int], num_tokens: int, allocate: Callable[[], int]) -> list[int]:
    """fork_block_table + the copy-on-write of the model's caches."""
    table, copies = fork_block_table(block_table, num_tokens, model.block_size, allocate)
    copy_blocks(model.k_cache, model.v_cache, copies)
    return table
