"""Numpy restatement of ``PagedCausalLM`` (engine/model.py:73-193).

TEST INFRASTRUCTURE ONLY — see oracle/__init__.py.

The weights come from an HF-named float32 state dict (the same dict the
reference's loader reads at engine/model.py:101-137). With
``quantize=True`` every layer linear is stored as (int8, scale) from
``quantize_per_channel`` and dequantized on each use, as the reference's
``QuantizedWeight.get()`` does; embeddings, norms, biases and the lm_head stay
float32 (engine/model.py:104-106, 127-137).
"""

from __future__ import annotations

import time

import numpy as np

from . import ops

F32 = np.float32

_LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


class OracleCausalLM:
    def __init__(self, state_dict: dict, shape, quantize: bool = True, max_position: int | None = None):
        self.shape = shape
        self.quantize = quantize
        self.H = shape.hidden
        self.Hq = shape.num_heads
        self.Hkv = shape.num_kv_heads
        self.D = shape.head_dim
        self.eps = shape.rms_eps
        self.embed = np.asarray(state_dict["model.embed_tokens.weight"], F32)
        self.final_norm = np.asarray(state_dict["model.norm.weight"], F32)
        self.lm_head = np.asarray(state_dict.get("lm_head.weight", self.embed), F32)
        self.layers = []
        for i in range(shape.num_layers):
            p = f"model.layers.{i}."
            lw = {
                "input_ln": np.asarray(state_dict[p + "input_layernorm.weight"], F32),
                "post_ln": np.asarray(state_dict[p + "post_attention_layernorm.weight"], F32),
            }
            for n in ("q", "k", "v"):
                b = state_dict.get(p + f"self_attn.{n}_proj.bias")
                lw[n + "_b"] = None if b is None else np.asarray(b, F32)
            for n in _LINEARS:
                sub = "self_attn" if n in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
                w = np.asarray(state_dict[p + f"{sub}.{n}.weight"], F32)
                lw[n] = ops.quantize_per_channel(w) if quantize else w
            self.layers.append(lw)
        mp = max_position or shape.max_position
        self.cos, self.sin = ops.build_rope_cache(mp, self.D, shape.rope_theta)
        self.k_cache = None
        self.v_cache = None
        self.block_size = None

    def _lin(self, x, w, b=None):
        if self.quantize:
            q, s = w
            return ops.quantized_linear(x, q, s, b)
        return ops.linear(x, w, b)

    def allocate_kv_cache(self, num_blocks: int, block_size: int) -> None:
        """engine/model.py:143-147: (L, NB, bs, Hkv, D) zeros."""
        shape = (len(self.layers), num_blocks, block_size, self.Hkv, self.D)
        self.k_cache = np.zeros(shape, F32)
        self.v_cache = np.zeros(shape, F32)
        self.block_size = block_size

    def forward_step(self, input_ids, block_table, start_pos: int, logits_rows=None, timings=None):
        """engine/model.py:149-193. Returns (T, V) float32 logits; when
        ``logits_rows`` is given only those rows of the lm_head product are
        computed (every other step is unchanged). ``timings`` (a dict), when
        given, accumulates wall seconds spent in the layer loop ("layers")
        and in embedding + final norm + lm_head ("head")."""
        t0 = time.perf_counter()
        ids = np.asarray(input_ids, np.int64)
        T = ids.shape[0]
        x = self.embed[ids]
        cos = self.cos[start_pos:start_pos + T]
        sin = self.sin[start_pos:start_pos + T]
        t1 = time.perf_counter()
        for li, lw in enumerate(self.layers):
            residual = x
            h = ops.rms_norm(x, lw["input_ln"], self.eps)
            q = self._lin(h, lw["q_proj"], lw["q_b"]).reshape(T, self.Hq, self.D)
            k = self._lin(h, lw["k_proj"], lw["k_b"]).reshape(T, self.Hkv, self.D)
            v = self._lin(h, lw["v_proj"], lw["v_b"]).reshape(T, self.Hkv, self.D)
            q = ops.apply_rope(q, cos, sin)
            k = ops.apply_rope(k, cos, sin)
            ops.write_kv(self.k_cache[li], self.v_cache[li], block_table, self.block_size, start_pos, k, v)
            a = ops.paged_causal_attention_incremental(
                q, self.k_cache[li], self.v_cache[li], block_table, self.block_size, start_pos)
            x = residual + self._lin(a.reshape(T, self.Hq * self.D), lw["o_proj"])
            residual = x
            h = ops.rms_norm(x, lw["post_ln"], self.eps)
            g = self._lin(h, lw["gate_proj"])
            u = self._lin(h, lw["up_proj"])
            x = residual + self._lin(ops.silu(g) * u, lw["down_proj"])
        t2 = time.perf_counter()
        x = ops.rms_norm(x, self.final_norm, self.eps)
        if logits_rows is not None:
            x = x[np.asarray(logits_rows)]
        out = ops.linear(x, self.lm_head)
        if timings is not None:
            t3 = time.perf_counter()
            timings["layers"] = timings.get("layers", 0.0) + (t2 - t1)
            timings["head"] = timings.get("head", 0.0) + (t1 - t0) + (t3 - t2)
        return out
