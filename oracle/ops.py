"""Numpy restatement of the reference's hot-path operators (float32 math).

TEST INFRASTRUCTURE ONLY — see oracle/__init__.py. Each function follows the
reference function named in its docstring, step for step, so that a mismatch
against the CUDA path is a bug in the CUDA path.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------- paging ----

def slot_of(block_table, block_size: int, pos: int) -> tuple[int, int]:
    """(physical block, offset) of logical position ``pos``:
    engine/paged_attention.py:74-77 (``block_idx = pos // bs``,
    ``offset = pos % bs``, ``phys = block_table[block_idx]``). A short table
    raises IndexError exactly like the reference's list indexing."""
    return block_table[pos // block_size], pos % block_size


def write_kv(k_cache, v_cache, block_table, block_size, start_pos, k, v) -> None:
    """engine/paged_attention.py:62-79. In place; dtype-agnostic (a plain row
    copy, so it is bit-exact on bf16 bit patterns held as uint16)."""
    for i in range(k.shape[0]):
        phys, off = slot_of(block_table, block_size, start_pos + i)
        k_cache[phys, off] = k[i]
        v_cache[phys, off] = v[i]


def gather_kv(k_cache, v_cache, block_table, block_size, seq_len):
    """engine/paged_attention.py:82-99: concatenate the first ``seq_len``
    logical rows out of the scattered blocks (partial last block via take)."""
    n_blocks = (seq_len + block_size - 1) // block_size
    ks, vs = [], []
    for b in range(n_blocks):
        phys = block_table[b]
        take = min(block_size, seq_len - b * block_size)
        ks.append(k_cache[phys, :take])
        vs.append(v_cache[phys, :take])
    return np.concatenate(ks, axis=0), np.concatenate(vs, axis=0)


# ------------------------------------------------------------- attention ----

def causal_attention_incremental(q, k, v, query_start_pos: int = 0):
    """engine/paged_attention.py:16-50. q (T, Hq, D); k, v (L, Hkv, D) with
    L = query_start_pos + T. GQA maps q head h to kv head h // (Hq // Hkv)
    (repeat_interleave, :36-37); scale 1/sqrt(D) (:40-41); key positions
    greater than the query's absolute position are masked (:43-46)."""
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    v = np.asarray(v, F32)
    T, Hq, D = q.shape
    L, Hkv, _ = k.shape
    group = Hq // Hkv
    k_ = np.repeat(k, group, axis=1).transpose(1, 0, 2)  # (Hq, L, D)
    v_ = np.repeat(v, group, axis=1).transpose(1, 0, 2)
    q_ = q.transpose(1, 0, 2)  # (Hq, T, D)
    scale = F32(1.0 / math.sqrt(D))
    scores = np.matmul(q_, k_.transpose(0, 2, 1)) * scale  # (Hq, T, L)
    qpos = np.arange(query_start_pos, query_start_pos + T)[:, None]
    kpos = np.arange(L)[None, :]
    scores = np.where(kpos > qpos, F32(-np.inf), scores)
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    p /= p.sum(axis=-1, keepdims=True)
    out = np.matmul(p.astype(F32), v_)  # (Hq, T, D)
    return out.transpose(1, 0, 2).astype(F32)


def reference_causal_attention(q, k, v):
    """engine/paged_attention.py:53-59."""
    return causal_attention_incremental(q, k, v, 0)


def paged_causal_attention(q, k_cache, v_cache, block_table, block_size, seq_len):
    """engine/paged_attention.py:102-114."""
    k, v = gather_kv(k_cache, v_cache, block_table, block_size, seq_len)
    return reference_causal_attention(q, k, v)


def paged_causal_attention_incremental(q_new, k_cache, v_cache, block_table, block_size, start_pos):
    """engine/paged_attention.py:117-132."""
    total = start_pos + q_new.shape[0]
    k, v = gather_kv(k_cache, v_cache, block_table, block_size, total)
    return causal_attention_incremental(q_new, k, v, start_pos)


# ---------------------------------------------------------- quantization ----

def quantize_per_channel(weight):
    """engine/quantization.py:16-23: absmax over K clamped to >= 1e-8,
    scale = absmax / 127 (float32, shape (N, 1)), q = clamp(round(w / scale),
    -127, 127) as int8. ``np.rint`` rounds half to even like ``torch.round``."""
    w = np.asarray(weight, F32)
    absmax = np.maximum(np.abs(w).max(axis=1, keepdims=True), F32(1e-8)).astype(F32)
    scale = (absmax / F32(127.0)).astype(F32)
    q = np.clip(np.rint(w / scale), -127, 127).astype(np.int8)
    return q, scale


def dequantize(q, scale):
    """engine/quantization.py:26-27 in float32 (``q.float() * scale``)."""
    return q.astype(F32) * scale.astype(F32)


def linear(x, w, b=None):
    """``F.linear(x, w, b)`` = x @ w.T + b (engine/model.py:168-193)."""
    y = np.asarray(x, F32) @ np.asarray(w, F32).T
    if b is not None:
        y = y + np.asarray(b, F32)
    return y.astype(F32)


def quantized_linear(x, q, scale, b=None):
    """``F.linear(x, QuantizedWeight.get(), b)`` (engine/model.py:25-26,
    engine/quantization.py:40-41): the weight is dequantized on every call,
    then a dense matmul."""
    return linear(x, dequantize(q, scale), b)


# ---------------------------------------------------------- norm / rope ----

def rms_norm(x, weight, eps):
    """engine/model.py:29-34 (float32 throughout)."""
    x = np.asarray(x, F32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    y = x * (F32(1.0) / np.sqrt(var + F32(eps)))
    return (np.asarray(weight, F32) * y).astype(F32)


def build_rope_cache(max_len, head_dim, theta):
    """engine/model.py:42-47: inv_freq = 1 / theta^(2i/D), emb =
    cat(freqs, freqs); returns float32 (cos, sin) of shape (max_len, D)."""
    inv_freq = (1.0 / (F32(theta) ** (np.arange(0, head_dim, 2, dtype=F32) / F32(head_dim)))).astype(F32)
    t = np.arange(max_len, dtype=F32)
    freqs = np.outer(t, inv_freq).astype(F32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def rotate_half(x):
    """engine/model.py:37-39."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_rope(x, cos, sin):
    """engine/model.py:50-54: x (T, H, D), cos/sin (T, D)."""
    return (x * cos[:, None, :] + rotate_half(x) * sin[:, None, :]).astype(F32)


def silu(x):
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


# ------------------------------------------------------- tensor parallel ----

def column_parallel_linear(x, full_weight, rank, world_size):
    """engine/tensor_parallel.py:21-31 (raises AssertionError on an uneven
    split, like the reference)."""
    n = full_weight.shape[0]
    assert n % world_size == 0, "output dim must divide evenly across ranks"
    s = n // world_size
    return np.asarray(x, F32) @ np.asarray(full_weight[rank * s:(rank + 1) * s], F32).T


def row_parallel_partial(x_shard, full_weight, rank, world_size):
    """engine/tensor_parallel.py:34-46: this rank's partial product before the
    all-reduce at :47."""
    k = full_weight.shape[1]
    assert k % world_size == 0, "input dim must divide evenly across ranks"
    s = k // world_size
    return np.asarray(x_shard, F32) @ np.asarray(full_weight[:, rank * s:(rank + 1) * s], F32).T


def row_parallel_linear_all_ranks(x_shards, full_weight):
    """engine/tensor_parallel.py:34-48 for every rank at once: the SUM
    all-reduce of the per-rank partials (every rank ends with this value)."""
    ws = len(x_shards)
    return sum(row_parallel_partial(x_shards[r], full_weight, r, ws) for r in range(ws)).astype(F32)


# ---------------------------------------------------------------- bf16 ----

def to_bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even (the
    conversion torch and CUDA's __float2bfloat16_rn perform)."""
    u = np.asarray(x, F32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, F32))
    out[nan] = 0x7FC0
    return out


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(F32)


def round_bf16(x) -> np.ndarray:
    return from_bf16_bits(to_bf16_bits(x))
