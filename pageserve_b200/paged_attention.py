"""Drop-in for the reference's engine/paged_attention.py, on sm_100a kernels.

Same function names, argument order and meaning; the tensors must be CUDA
tensors (bf16 or f16 for attention). ``block_table`` may be a Python list
(as in the reference) or an int32 CUDA tensor (the graph-capturable form).
A block table too short for the requested positions raises IndexError, as
the reference's list indexing does (engine/paged_attention.py:77, 95).

Batched entry point beyond the reference: :func:`paged_attention` runs many
sequences (decode and chunked prefill) in one launch from device-resident
metadata.
"""

from __future__ import annotations

import math

import torch

from . import _lib


def _table_tensor(block_table, device) -> torch.Tensor:
    if isinstance(block_table, torch.Tensor):
        t = block_table.to(device=device, dtype=torch.int32)
        return t.contiguous()
    return torch.tensor(list(block_table), dtype=torch.int32, device=device)


def _table_len(block_table) -> int:
    return int(block_table.numel()) if isinstance(block_table, torch.Tensor) else len(block_table)


def write_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, block_table, block_size: int, start_pos: int,
             k: torch.Tensor, v: torch.Tensor) -> None:
    """engine/paged_attention.py:62-79: write k[i], v[i] (positions
    start_pos + i) into slot block_table[pos // bs] * bs + pos % bs. In place,
    bit-exact."""
    _lib.require_cuda(k_cache, v_cache, k, v)
    if k_cache.dtype != k.dtype or v_cache.dtype != v.dtype:
        raise TypeError("write_kv: cache and k/v dtypes differ")
    nb, bs, hkv, d = k_cache.shape
    if bs != block_size:
        raise ValueError(f"write_kv: cache block size {bs} != block_size {block_size}")
    T = k.shape[0]
    if T == 0:
        return
    n_needed = (start_pos + T - 1) // block_size + 1
    if _table_len(block_table) < n_needed:
        raise IndexError(f"block_table has {_table_len(block_table)} entries; position {start_pos + T - 1} "
                         f"needs {n_needed}")
    table = _table_tensor(block_table, k_cache.device)
    k = k.contiguous()
    v = v.contiguous()
    lib = _lib.load()
    _lib.check(lib.ps_write_kv(k_cache.data_ptr(), v_cache.data_ptr(), table.data_ptr(), table.numel(), nb,
                               block_size, hkv, d, _lib.dtype_code(k.dtype), start_pos, T, k.data_ptr(),
                               v.data_ptr(), _lib.stream_ptr()), "write_kv")


def gather_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, block_table, block_size: int, seq_len: int):
    """engine/paged_attention.py:82-99 (a debugging/test utility: the kernels
    below never materialise the gathered copy)."""
    n = (seq_len + block_size - 1) // block_size
    if _table_len(block_table) < n:
        raise IndexError(f"block_table has {_table_len(block_table)} entries, {n} needed")
    table = _table_tensor(block_table, k_cache.device)[:n].long()
    pos = torch.arange(seq_len, device=k_cache.device)
    slots = table[pos // block_size] * block_size + pos % block_size
    flat_k = k_cache.reshape(-1, *k_cache.shape[2:])
    flat_v = v_cache.reshape(-1, *v_cache.shape[2:])
    return flat_k.index_select(0, slots), flat_v.index_select(0, slots)


class AttentionWorkspace:
    """Grow-only scratch buffer for split-context partials (reused across
    calls; allocate it before capturing a CUDA graph)."""

    def __init__(self):
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int, device) -> torch.Tensor | None:
        if nbytes == 0:
            return None
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != torch.device(device):
            self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return self.buf


_default_ws: dict[torch.device, AttentionWorkspace] = {}


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                    cu_q: torch.Tensor, start_pos: torch.Tensor, max_q_len: int, max_ctx: int,
                    out: torch.Tensor | None = None, workspace: AttentionWorkspace | None = None) -> torch.Tensor:
    """Batched paged attention. q (total_q, Hq, D); caches (NB, bs, Hkv, D);
    block_tables int32 (B, max_blocks); cu_q int32 (B+1,) cumulative query
    counts; start_pos int32 (B,). Sequence b's query i sits at absolute
    position start_pos[b] + i and attends causally to its context
    (engine/paged_attention.py:16-50, 117-132)."""
    _lib.require_cuda(q, k_cache, v_cache, block_tables, cu_q, start_pos)
    total_q, hq, d = q.shape
    nb, bs, hkv, d2 = k_cache.shape
    if d2 != d or v_cache.shape != k_cache.shape:
        raise ValueError("paged_attention: cache / query head_dim mismatch")
    if q.dtype != k_cache.dtype:
        raise TypeError("paged_attention: q and cache dtypes differ")
    for t in (block_tables, cu_q, start_pos):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise TypeError("paged_attention: metadata must be contiguous int32")
    B = start_pos.numel()
    q = q.contiguous()
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    ws_bytes = lib.ps_paged_attention_workspace_size(B, max_q_len, max_ctx, hq, hkv, d)
    if workspace is None:
        workspace = _default_ws.setdefault(q.device, AttentionWorkspace())
    buf = workspace.get(ws_bytes, q.device)
    _lib.check(lib.ps_paged_attention(out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                      block_tables.data_ptr(), block_tables.shape[-1], cu_q.data_ptr(),
                                      start_pos.data_ptr(), B, total_q, max_q_len, max_ctx, nb, bs, hq, hkv, d,
                                      _lib.dtype_code(q.dtype), _lib.ptr(buf), ws_bytes, _lib.stream_ptr()),
               "paged_attention")
    return out


def paged_causal_attention_incremental(q_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                       block_table, block_size: int, start_pos: int) -> torch.Tensor:
    """engine/paged_attention.py:117-132: q_new covers this step's chunk;
    its K/V must already be in the cache (write_kv)."""
    _lib.require_cuda(q_new, k_cache, v_cache)
    T = q_new.shape[0]
    total = start_pos + T
    n = (total + block_size - 1) // block_size
    if _table_len(block_table) < n:
        raise IndexError(f"block_table has {_table_len(block_table)} entries; context {total} needs {n}")
    if k_cache.shape[1] != block_size:
        raise ValueError("cache block size mismatch")
    dev = q_new.device
    table = _table_tensor(block_table, dev).reshape(1, -1)
    meta = torch.tensor([0, T, start_pos], dtype=torch.int32, device=dev)
    return paged_attention(q_new, k_cache, v_cache, table, meta[0:2], meta[2:3], T, total)


def causal_attention_incremental(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 query_start_pos: int = 0) -> torch.Tensor:
    """engine/paged_attention.py:16-50 on contiguous K/V: the (L, Hkv, D)
    tensors are one cache block of size L, read by the same kernel."""
    L = k.shape[0]
    kc = k.contiguous().reshape(1, L, *k.shape[1:])
    vc = v.contiguous().reshape(1, L, *v.shape[1:])
    return paged_causal_attention_incremental(q, kc, vc, [0], L, query_start_pos)


def reference_causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """engine/paged_attention.py:53-59."""
    return causal_attention_incremental(q, k, v, 0)


def paged_causal_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table,
                           block_size: int, seq_len: int) -> torch.Tensor:
    """engine/paged_attention.py:102-114 (full prefill from position 0)."""
    if q.shape[0] != seq_len:
        raise ValueError("paged_causal_attention: q must cover the whole sequence")
    return paged_causal_attention_incremental(q, k_cache, v_cache, block_table, block_size, 0)


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
