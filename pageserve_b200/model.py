"""Drop-in for the reference's engine/model.py on the sm_100a kernels.

``PagedCausalLM`` keeps the reference's constructor, ``allocate_kv_cache``,
``forward_step`` and attributes (``device``, ``dtype``, ``config``,
``layers``, ``k_cache``, ``v_cache``, ``block_size``, ...), and adds
``forward_batch`` — one pass over a whole scheduler step (many decode
sequences plus chunked-prefill chunks) from device-resident block tables —
and ``capture_decode_graph`` for CUDA-graph replay of a decode step.

Per layer the step runs (engine/model.py:164-190):
  rmsnorm -> fused QKV W8A16 linear (+bias) -> RoPE + KV-slot write ->
  paged attention -> o_proj W8A16 (+residual) -> rmsnorm ->
  fused gate|up W8A16 -> SiLU*up -> down_proj W8A16 (+residual)
then the final rmsnorm, the bf16 lm_head and an on-device argmax.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from types import SimpleNamespace

import numpy as np
import torch

from . import _lib
from .batch import attention_runs, pack_metadata
from .paged_attention import AttentionWorkspace, paged_attention
from .quantization import LinearWorkspace, QuantizedWeight, RowView, linear16, linear_swiglu

Weight = torch.Tensor | QuantizedWeight


# ------------------------------------------------------- reference ops ----

def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """engine/model.py:29-34 as one fused kernel (float32 math)."""
    return rms_norm_fused(x, weight, eps)


def rms_norm_fused(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
                   residual_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = rmsnorm(x [+ residual]) * weight; the sum is also stored to
    residual_out when given (engine/model.py:29-34, 184, 190). Replaces the
    reference's Triton kernel (kernels/rmsnorm_triton.py:46-57)."""
    _lib.require_cuda(x, weight, residual)
    H = x.shape[-1]
    x2 = x.reshape(-1, H).contiguous()
    if out is None:
        out = torch.empty_like(x2)
    w = weight.to(x.dtype).contiguous()
    r = None if residual is None else residual.reshape(-1, H).contiguous()
    _lib.check(_lib.load().ps_rmsnorm(out.data_ptr(), _lib.ptr(residual_out), x2.data_ptr(), _lib.ptr(r),
                                      w.data_ptr(), float(eps), x2.shape[0], H, _lib.dtype_code(x.dtype),
                                      _lib.stream_ptr(x.device)), "rmsnorm")
    return out.reshape(x.shape)


# The reference's Triton entry point name (kernels/rmsnorm_triton.py:46).
rms_norm_triton = rms_norm


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """engine/model.py:37-39."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def build_rope_cache(max_len: int, head_dim: int, theta: float, device, dtype):
    """engine/model.py:42-47 (init-time table)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    t = torch.arange(max_len, device=device).float()
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def build_rope_table_f32(max_len: int, head_dim: int, theta: float, device):
    """float32 (max_len, head_dim/2) cos/sin halves for the fused RoPE kernel
    (same formula as engine/model.py:42-47, kept in float32)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    t = torch.arange(max_len, device=device).float()
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().contiguous(), freqs.sin().contiguous()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """engine/model.py:50-54: x (T, H, D), cos/sin (T, D)."""
    _lib.require_cuda(x, cos, sin)
    T, H, D = x.shape
    x = x.contiguous()
    out = torch.empty_like(x)
    c = cos.to(x.dtype).contiguous()
    s = sin.to(x.dtype).contiguous()
    _lib.check(_lib.load().ps_apply_rope(out.data_ptr(), x.data_ptr(), c.data_ptr(), s.data_ptr(), T, H, D,
                                         _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device)), "apply_rope")
    return out


@dataclass
class LayerWeights:
    """engine/model.py:57-70."""
    input_ln: torch.Tensor
    post_ln: torch.Tensor
    q_w: Weight
    k_w: Weight
    v_w: Weight
    o_w: Weight
    gate_w: Weight
    up_w: Weight
    down_w: Weight
    q_b: torch.Tensor | None = None
    k_b: torch.Tensor | None = None
    v_b: torch.Tensor | None = None


@dataclass
class FusedLayer:
    """Kernel-side layout of one layer: projections sharing an input are
    concatenated along N (per-channel scales make this exact)."""
    input_ln: torch.Tensor
    post_ln: torch.Tensor
    qkv: Weight
    qkv_b: torch.Tensor
    o: Weight
    gate_up: Weight  # rows interleaved: 2i = gate row i, 2i+1 = up row i (the SwiGLU linear's layout)
    down: Weight


def _cat_weights(ws: list[Weight], dtype) -> Weight:
    if isinstance(ws[0], QuantizedWeight):
        return QuantizedWeight.from_quantized(torch.cat([w.q for w in ws], 0), torch.cat([w.scale for w in ws], 0),
                                              dtype)
    return torch.cat(ws, 0).contiguous()


def _interleave_rows(a: Weight, b: Weight, dtype) -> Weight:
    """Rows a0, b0, a1, b1, ... (per-row scales travel with their rows, so
    this is exact for int8 weights)."""
    def il(x, y):
        return torch.stack([x, y], dim=1).reshape(2 * x.shape[0], *x.shape[1:]).contiguous()
    if isinstance(a, QuantizedWeight):
        return QuantizedWeight.from_quantized(il(a.q, b.q), il(a.scale, b.scale), dtype)
    return il(a, b)


def _one_copy(lw: "LayerWeights", fl: "FusedLayer", dtype) -> None:
    """Keep one int8 copy of each of a layer's weights in HBM: the kernels'
    tiled copies (built here, before any graph capture). The reference-facing
    per-projection weights become row views of the fused q|k|v and gate|up
    weights and the row-major copies are dropped (``q`` is rebuilt from the
    tiled copy on access, outside the hot path). Done layer by layer so
    loading never holds more than one layer's extra copies."""
    for w in (fl.qkv, fl.o, fl.gate_up, fl.down):
        if isinstance(w, QuantizedWeight):
            w.release_row_major()
    if isinstance(fl.qkv, QuantizedWeight):
        nq, nk = lw.q_w.shape[0], lw.k_w.shape[0]
        lw.q_w = RowView(fl.qkv, slice(0, nq), dtype)
        lw.k_w = RowView(fl.qkv, slice(nq, nq + nk), dtype)
        lw.v_w = RowView(fl.qkv, slice(nq + nk, nq + 2 * nk), dtype)
    if isinstance(fl.gate_up, QuantizedWeight):
        lw.gate_w = RowView(fl.gate_up, slice(0, None, 2), dtype)
        lw.up_w = RowView(fl.gate_up, slice(1, None, 2), dtype)


def two_shot_ok(world: int, hidden: int) -> bool:
    """The two-shot reduction scatters whole 128-column output tiles."""
    return world > 1 and hidden % world == 0 and (hidden // world) % 128 == 0


def auto_tp_comm(world: int, hidden: int) -> str:
    """Row-parallel reduction transport for ``tp_comm="auto"``, by measurement
    on B200s (config-4 step, 576 tokens x 2048): at 2 ranks the one-shot push
    (one peer, one synchronisation); from 4 ranks NCCL (4 ranks: 5.72 ms per
    step vs one-shot 6.07 ms vs two-shot 8.54 ms). The exchanges are
    latency-bound at these sizes (0.26-2.4 MB), so the two-shot's second
    synchronisation stage costs more than the bytes it saves."""
    return "fused" if world <= 2 else "nccl"


def _check_device_dtype(device, dtype) -> None:
    if torch.device(device).type != "cuda":
        raise RuntimeError("pageserve_b200.PagedCausalLM runs on CUDA only (no CPU fallback); pass device='cuda'")
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"pageserve_b200.PagedCausalLM computes in bfloat16 or float16, not {dtype}")


class StepMeta:
    """Device-resident metadata of one step (int32)."""

    def __init__(self, block_tables: torch.Tensor, cu_q: torch.Tensor, start_pos: torch.Tensor, q_lens: list[int],
                 ctx_lens: list[int]):
        self.block_tables = block_tables
        self.cu_q = cu_q
        self.start_pos = start_pos
        self.q_lens = q_lens
        self.ctx_lens = ctx_lens


class PagedCausalLM:
    """engine/model.py:73-193 on the sm_100a kernels."""

    def __init__(self, model_id: str, device: str = "cpu", dtype: torch.dtype = torch.float32,
                 quantize: bool = False):
        """engine/model.py:77-141, same arguments and defaults. This build runs
        on CUDA only, in bfloat16 or float16: the reference's CPU / float32
        defaults raise RuntimeError / ValueError (no CPU fallback), so a caller
        passes ``device="cuda", dtype=torch.bfloat16`` as the reference's own
        GPU callers do (server.py:40, app.py:80). Like the reference, the
        checkpoint is loaded in ``dtype`` and quantized from it."""
        from transformers import AutoConfig, AutoModelForCausalLM

        _check_device_dtype(device, dtype)
        config = AutoConfig.from_pretrained(model_id)
        hf = AutoModelForCausalLM.from_pretrained(model_id, torch_dtype=dtype)
        sd = hf.state_dict()
        del hf
        rope_params = getattr(config, "rope_parameters", None)
        theta = rope_params["rope_theta"] if rope_params else config.rope_theta
        self._init(config, sd, device, dtype, quantize, theta)

    @classmethod
    def from_state_dict(cls, state_dict: dict, shape, device: str = "cuda", dtype: torch.dtype = torch.bfloat16,
                        quantize: bool = True, max_position: int | None = None, tp=None, tp_comm: str = "auto",
                        tp_max_tokens: int = 4096) -> "PagedCausalLM":
        """Build from an HF-named state dict (numpy or torch tensors) and a
        ``synthetic.Qwen2Shape`` (the seeded random-init checkpoints). With
        ``tp`` (a ``tensor_parallel.TPGroup``) this rank loads only its
        Megatron shard (engine/tensor_parallel.py). ``tp_comm`` picks the
        row-parallel reduction: "fused" (one-shot peer-memory push from the
        linear into the next RMSNorm, at most ``tp_max_tokens`` tokens per
        step), "fused2" (two-shot: the linear scatters column slices to their
        owner ranks, which reduce, all-gather the residual stream and
        normalise), "nccl" (torch.distributed all_reduce, the reference's
        collective) or "auto" (``auto_tp_comm``)."""
        cfg = SimpleNamespace(num_attention_heads=shape.num_heads, num_key_value_heads=shape.num_kv_heads,
                              hidden_size=shape.hidden, head_dim=shape.head_dim, rms_norm_eps=shape.rms_eps,
                              rope_theta=shape.rope_theta, rope_parameters=None,
                              max_position_embeddings=max_position or shape.max_position,
                              num_hidden_layers=shape.num_layers, vocab_size=shape.vocab,
                              intermediate_size=shape.intermediate, tie_word_embeddings=shape.tie_embeddings)
        obj = cls.__new__(cls)
        obj._init(cfg, state_dict, device, dtype, quantize, shape.rope_theta, tp, tp_comm, tp_max_tokens)
        return obj

    def _init(self, config, sd, device, dtype, quantize, theta, tp=None, tp_comm="auto", tp_max_tokens=4096):
        _check_device_dtype(device, dtype)
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        _lib.load()
        _lib.ensure_status_word(self.device)
        self.dtype = dtype
        self.quantize = quantize
        self.config = config
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.hidden_size = config.hidden_size
        self.head_dim = getattr(config, "head_dim", None) or self.hidden_size // self.num_heads
        self.tp = tp if (tp is not None and tp.world > 1) else None
        self.shard = None
        if self.tp is not None:
            from .tensor_parallel import ShardPlan
            inter = config.intermediate_size if hasattr(config, "intermediate_size") else \
                int(sd["model.layers.0.mlp.gate_proj.weight"].shape[0])
            vocab = int(sd["model.embed_tokens.weight"].shape[0])
            self.shard = ShardPlan(self.tp.rank, self.tp.world, self.num_heads, self.num_kv_heads, self.head_dim,
                                   inter, vocab)
        self.rms_eps = config.rms_norm_eps
        self.rope_theta = theta
        self.max_position_embeddings = config.max_position_embeddings

        self.heads_local = self.shard.heads_local if self.shard else self.num_heads
        self.kv_heads_local = self.shard.kv_heads_local if self.shard else self.num_kv_heads

        def T(key):
            v = sd[key]
            return (torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else v)

        def dev(key, dt=None):
            return T(key).to(device=self.device, dtype=dt or dtype).contiguous()

        sp = self.shard

        def rows_of(key):
            """Column-parallel rows of this rank (None = all)."""
            if sp is None:
                return None
            if key.endswith(("q_proj.weight", "q_proj.bias")):
                return sp.q_rows()
            if key.endswith(("k_proj.weight", "v_proj.weight", "k_proj.bias", "v_proj.bias")):
                return sp.kv_rows()
            if key.endswith(("gate_proj.weight", "up_proj.weight")):
                return list(sp.inter_cols)
            return None

        def cols_of(key):
            """Row-parallel input columns of this rank (None = all)."""
            if sp is None:
                return None
            if key.endswith("o_proj.weight"):
                return sp.q_rows()
            if key.endswith("down_proj.weight"):
                return list(sp.inter_cols)
            return None

        def load_weight(key) -> Weight:
            w = T(key).to(self.device)
            rows, cols = rows_of(key), cols_of(key)
            if rows is not None:  # row slices quantize identically (per-row scales)
                w = w[torch.as_tensor(rows, device=w.device)]
            if quantize:
                qw = QuantizedWeight(w)
                qw.dtype = dtype
                if cols is not None:  # keep the full-row scale: partials sum to the unsharded linear
                    qw.q = qw.q[:, torch.as_tensor(cols, device=w.device)].contiguous()
                return qw
            if cols is not None:
                w = w[:, torch.as_tensor(cols, device=w.device)]
            return w.to(dtype).contiguous()

        def bias(key):
            if key not in sd:
                return None
            b = T(key).to(self.device)
            rows = rows_of(key)
            if rows is not None:
                b = b[torch.as_tensor(rows, device=b.device)]
            return b.to(dtype).contiguous()

        self.embed_tokens = dev("model.embed_tokens.weight")
        self.final_norm_w = dev("model.norm.weight")
        lm = dev("lm_head.weight") if "lm_head.weight" in sd else self.embed_tokens
        self.vocab_offset = 0
        if sp is not None:
            vr = sp.vocab_rows
            lm = lm[vr.start:vr.stop].contiguous()
            self.vocab_offset = vr.start
        self.lm_head_w = lm
        self.layers: list[LayerWeights] = []
        self.fused: list[FusedLayer] = []
        for i in range(config.num_hidden_layers):
            p = f"model.layers.{i}."
            lw = LayerWeights(
                input_ln=dev(p + "input_layernorm.weight"),
                post_ln=dev(p + "post_attention_layernorm.weight"),
                q_w=load_weight(p + "self_attn.q_proj.weight"),
                k_w=load_weight(p + "self_attn.k_proj.weight"),
                v_w=load_weight(p + "self_attn.v_proj.weight"),
                o_w=load_weight(p + "self_attn.o_proj.weight"),
                gate_w=load_weight(p + "mlp.gate_proj.weight"),
                up_w=load_weight(p + "mlp.up_proj.weight"),
                down_w=load_weight(p + "mlp.down_proj.weight"),
                q_b=bias(p + "self_attn.q_proj.bias"),
                k_b=bias(p + "self_attn.k_proj.bias"),
                v_b=bias(p + "self_attn.v_proj.bias"),
            )
            self.layers.append(lw)
            hq, hkv, d = self.heads_local, self.kv_heads_local, self.head_dim
            zb = lambda n: torch.zeros(n, dtype=dtype, device=self.device)  # noqa: E731
            qkv_b = torch.cat([lw.q_b if lw.q_b is not None else zb(hq * d),
                               lw.k_b if lw.k_b is not None else zb(hkv * d),
                               lw.v_b if lw.v_b is not None else zb(hkv * d)]).contiguous()
            self.fused.append(FusedLayer(
                input_ln=lw.input_ln, post_ln=lw.post_ln,
                qkv=_cat_weights([lw.q_w, lw.k_w, lw.v_w], dtype), qkv_b=qkv_b, o=lw.o_w,
                gate_up=_interleave_rows(lw.gate_w, lw.up_w, dtype), down=lw.down_w))
            _one_copy(lw, self.fused[-1], dtype)

        self.intermediate_size = (self.layers[0].gate_w.shape[0] if self.layers else 0)  # local under TP
        self.vocab_size = self.embed_tokens.shape[0]
        self.cos_cache, self.sin_cache = build_rope_cache(self.max_position_embeddings, self.head_dim, theta,
                                                          self.device, dtype)
        self.rope_cos, self.rope_sin = build_rope_table_f32(self.max_position_embeddings, self.head_dim, theta,
                                                            self.device)
        self.attn_ws = AttentionWorkspace()
        # Prefill and decode attention of one step are independent (disjoint
        # output rows, read-only q and caches): the prefill runs go to a side
        # stream (own workspace) so their small grid overlaps the HBM-bound
        # decode kernel; PS_ATTN_CONCURRENT=0 runs them back to back.
        self.attn_ws_side = AttentionWorkspace()
        self._attn_side = torch.cuda.Stream(device=self.device)
        self._attn_concurrent = os.environ.get("PS_ATTN_CONCURRENT", "1") != "0"
        self.lin_ws = LinearWorkspace()
        if tp_comm not in ("fused", "fused2", "nccl", "auto"):
            raise ValueError(f"tp_comm must be 'fused', 'fused2', 'nccl' or 'auto', not {tp_comm!r}")
        if tp_comm == "auto":
            tp_comm = auto_tp_comm(self.tp.world if self.tp is not None else 1, self.hidden_size)
        if tp_comm == "fused2" and self.tp is not None and not two_shot_ok(self.tp.world, self.hidden_size):
            raise ValueError(f"tp_comm='fused2' needs hidden/world a multiple of 128 "
                             f"(hidden {self.hidden_size}, world {self.tp.world})")
        self.tp_comm = tp_comm if self.tp is not None else None
        self.comm = None
        if self.tp is not None and tp_comm in ("fused", "fused2"):
            from .comm import FusedAllReduce
            self.comm = FusedAllReduce.create(self.tp.rank, self.tp.world, tp_max_tokens, self.hidden_size, dtype,
                                              self.device, self.tp.group)
        self.k_cache = None
        self.v_cache = None
        self.block_size = None

    # ------------------------------------------------------------ memory --
    def allocate_kv_cache(self, num_blocks: int, block_size: int) -> None:
        """engine/model.py:143-147: (L, NB, bs, Hkv, D) zeros."""
        shape = (len(self.layers), num_blocks, block_size, self.kv_heads_local, self.head_dim)
        self.k_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.block_size = block_size
        self.num_blocks = num_blocks

    # ------------------------------------------------------------- linear --
    def _linear(self, x, w: Weight, bias=None, residual=None):
        if isinstance(w, QuantizedWeight):
            return w.linear(x, bias, residual, workspace=self.lin_ws)
        return linear16(x, w, bias, residual, workspace=self.lin_ws)

    # -------------------------------------------------------------- steps --
    def make_meta(self, q_lens: list[int], start_pos: list[int], block_tables: list[list[int]],
                  max_blocks: int | None = None) -> StepMeta:
        """Host lists -> device int32 metadata (one host->device copy).
        Raises IndexError when a block table is too short for its context
        (engine/paged_attention.py:77) or names a block outside the pool."""
        buf, B, mb, ctx = pack_metadata(q_lens, start_pos, block_tables, self.block_size, self.num_blocks,
                                        max_blocks)
        d = torch.from_numpy(buf).to(self.device, non_blocking=False)
        return StepMeta(d[2 * B + 1:].view(B, mb), d[:B + 1], d[B + 1:2 * B + 1], list(q_lens), ctx)

    def _forward(self, ids: torch.Tensor, meta: StepMeta, logits_rows: torch.Tensor | None):
        T = ids.shape[0]
        H, hq, hkv, d = self.hidden_size, self.heads_local, self.kv_heads_local, self.head_dim
        lead = self.tp is None or self.tp.rank == 0  # adds the residual exactly once
        lib = _lib.load()
        stream = _lib.stream_ptr(self.device)
        x = torch.empty((T, H), dtype=self.dtype, device=self.device)
        _lib.check(lib.ps_embedding(x.data_ptr(), ids.data_ptr(), self.embed_tokens.data_ptr(), T, H,
                                    self.vocab_size, _lib.dtype_code(self.dtype), stream), "embedding")
        positions = torch.empty(T, dtype=torch.int32, device=self.device)
        slots = torch.empty(T, dtype=torch.int32, device=self.device)
        B = len(meta.q_lens)
        _lib.check(lib.ps_build_slot_mapping(positions.data_ptr(), slots.data_ptr(), meta.block_tables.data_ptr(),
                                             meta.block_tables.shape[1], meta.cu_q.data_ptr(),
                                             meta.start_pos.data_ptr(), B, T, self.num_blocks, self.block_size,
                                             stream), "build_slot_mapping")
        runs = attention_runs(meta.q_lens, hq // hkv)
        q = torch.empty((T, hq, d), dtype=self.dtype, device=self.device)
        attn = torch.empty((T, hq, d), dtype=self.dtype, device=self.device)
        num_slots = self.num_blocks * self.block_size
        comm = self.comm  # fused TP reduction: o_proj -> set 0, down_proj -> set 1, consumed by the next norm
        if comm is not None and T > comm.max_tokens:
            raise ValueError(f"{T} tokens exceed tp_max_tokens={comm.max_tokens}")
        if comm is not None and self.tp_comm == "fused2":
            return self._forward_two_shot(x, q, attn, positions, slots, meta, runs, logits_rows)
        pending = False  # a down_proj reduction waits in set 1
        for li, fl in enumerate(self.fused):
            if pending:
                h = comm.allreduce_rmsnorm(x, fl.input_ln, self.rms_eps, 1)
            else:
                h = rms_norm_fused(x, fl.input_ln, self.rms_eps)
            qkv = self._linear(h, fl.qkv, fl.qkv_b)
            kc, vc = self.k_cache[li], self.v_cache[li]
            _lib.check(lib.ps_rope_qkv_write_kv(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), qkv.data_ptr(),
                                                positions.data_ptr(), slots.data_ptr(), self.rope_cos.data_ptr(),
                                                self.rope_sin.data_ptr(), self.max_position_embeddings, T, hq, hkv,
                                                d, num_slots, _lib.dtype_code(self.dtype), stream), "rope_qkv")
            self._attention(q, kc, vc, meta, runs, attn)
            if comm is not None:
                comm.linear_push(attn.view(T, hq * d), fl.o, 0, workspace=self.lin_ws)
                h = comm.allreduce_rmsnorm(x, fl.post_ln, self.rms_eps, 0)
            else:
                x = self._linear(attn.view(T, hq * d), fl.o, residual=x if lead else None)
                if self.tp is not None:
                    self.tp.all_reduce_(x)
                h = rms_norm_fused(x, fl.post_ln, self.rms_eps)
            act = linear_swiglu(h, fl.gate_up)  # silu(gate) * up in the gate|up linear's epilogue
            if comm is not None:
                comm.linear_push(act, fl.down, 1, workspace=self.lin_ws)
                pending = True
            else:
                x = self._linear(act, fl.down, residual=x if lead else None)
                if self.tp is not None:
                    self.tp.all_reduce_(x)
        if pending:  # the last down_proj reduction, consumed by the final norm (all rows, then the selection)
            x = comm.allreduce_rmsnorm(x, self.final_norm_w, self.rms_eps, 1)
            if logits_rows is not None:
                x = x.index_select(0, logits_rows)
        else:
            if logits_rows is not None:
                x = x.index_select(0, logits_rows)
            x = rms_norm_fused(x, self.final_norm_w, self.rms_eps)
        return linear16(x, self.lm_head_w, workspace=self.lin_ws)

    def _forward_two_shot(self, x, q, attn, positions, slots, meta, runs, logits_rows):
        """The layer loop with the two-shot fused reduction: each row-parallel
        linear scatters its output's column slices to their owner ranks, whose
        reduce kernel adds the residual, all-gathers the new residual stream
        (kept in the receive buffer's gathered region) and normalises it for
        the next linear (engine/model.py:164-193 with the all-reduce of
        engine/tensor_parallel.py:47)."""
        T = x.shape[0]
        hq, hkv, d = self.heads_local, self.kv_heads_local, self.head_dim
        lib = _lib.load()
        stream = _lib.stream_ptr(self.device)
        comm = self.comm
        num_slots = self.num_blocks * self.block_size
        resid = x  # the residual stream: the embedding, then the gathered region of the last set reduced
        h = rms_norm_fused(x, self.fused[0].input_ln, self.rms_eps) if self.fused else None
        for li, fl in enumerate(self.fused):
            qkv = self._linear(h, fl.qkv, fl.qkv_b)
            kc, vc = self.k_cache[li], self.v_cache[li]
            _lib.check(lib.ps_rope_qkv_write_kv(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), qkv.data_ptr(),
                                                positions.data_ptr(), slots.data_ptr(), self.rope_cos.data_ptr(),
                                                self.rope_sin.data_ptr(), self.max_position_embeddings, T, hq, hkv,
                                                d, num_slots, _lib.dtype_code(self.dtype), stream), "rope_qkv")
            self._attention(q, kc, vc, meta, runs, attn)
            comm.linear_push(attn.view(T, hq * d), fl.o, 0, workspace=self.lin_ws, scatter=True)
            h = comm.reduce_norm(resid, fl.post_ln, self.rms_eps, 0, T)
            resid = comm.gathered_ptr(0)
            act = linear_swiglu(h, fl.gate_up)
            comm.linear_push(act, fl.down, 1, workspace=self.lin_ws, scatter=True)
            nxt = self.fused[li + 1].input_ln if li + 1 < len(self.fused) else self.final_norm_w
            h = comm.reduce_norm(resid, nxt, self.rms_eps, 1, T)
            resid = comm.gathered_ptr(1)
        if h is None:
            h = rms_norm_fused(x, self.final_norm_w, self.rms_eps)
        if logits_rows is not None:
            h = h.index_select(0, logits_rows)
        return linear16(h, self.lm_head_w, workspace=self.lin_ws)

    def _attention(self, q, kc, vc, meta, runs, attn) -> None:
        """Paged attention of every run into its rows of ``attn``; with both
        kinds present, the prefill runs on the side stream (forked after the
        KV write, joined before o_proj), launched first so its CTAs start
        before the decode grid fills the SMs."""
        def run(s, e, ws):
            paged_attention(q, kc, vc, meta.block_tables[s:e], meta.cu_q[s:e + 1], meta.start_pos[s:e],
                            max(meta.q_lens[s:e]), max(meta.ctx_lens[s:e]), out=attn, workspace=ws)
        kinds = {d for (_, _, d) in runs}
        if not (self._attn_concurrent and len(kinds) == 2):
            for (s, e, _) in runs:
                run(s, e, self.attn_ws)
            return
        main = torch.cuda.current_stream(self.device)
        side = self._attn_side
        fork, join = torch.cuda.Event(), torch.cuda.Event()
        fork.record(main)
        side.wait_event(fork)
        with torch.cuda.stream(side):
            for (s, e, dec) in runs:
                if not dec:
                    run(s, e, self.attn_ws_side)
        join.record(side)
        for (s, e, dec) in runs:
            if dec:
                run(s, e, self.attn_ws)
        main.wait_event(join)

    def close(self) -> None:
        """Release the fused all-reduce buffers and peer mappings (call on
        every rank before destroy_process_group)."""
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def forward_step(self, input_ids: torch.Tensor, block_table: list[int], start_pos: int) -> torch.Tensor:
        """engine/model.py:149-193: one chunk of one sequence; returns
        (chunk_len, vocab) logits."""
        if self.k_cache is None:
            raise RuntimeError("allocate_kv_cache() must run before forward_step()")
        ids = input_ids.to(device=self.device, dtype=torch.int64).reshape(-1)
        T = ids.shape[0]
        meta = self.make_meta([T], [int(start_pos)], [list(block_table)])
        return self.gather_logits(self._forward(ids, meta, None))

    def forward_batch(self, input_ids, q_lens: list[int], start_pos: list[int], block_tables: list[list[int]],
                      return_logits: bool = True, top_k: int | None = None, temperature: float = 1.0,
                      generator: torch.Generator | None = None):
        """One scheduler step for many sequences in one pass (superset of the
        reference, which calls forward_step once per sequence,
        engine/runner.py:65-79). input_ids: the chunks concatenated in
        sequence order. Returns (logits of each sequence's last token (B, V),
        next tokens int32 (B,)): greedy, or with ``top_k`` sampled on the
        device from softmax(top-k logits / temperature)."""
        if self.k_cache is None:
            raise RuntimeError("allocate_kv_cache() must run before forward_batch()")
        ids = torch.as_tensor(input_ids, dtype=torch.int64).to(self.device).reshape(-1)
        meta = self.make_meta(q_lens, start_pos, block_tables)
        last = meta.cu_q[1:].to(torch.int64) - 1
        logits = self._forward(ids, meta, last)
        if top_k is None:
            return (self.gather_logits(logits) if return_logits else None), self.next_tokens(logits)
        from .sampling import sample_top_k
        full = self.gather_logits(logits)
        nxt = sample_top_k(full, top_k, temperature, generator=generator)
        if self.tp is not None:  # every rank keeps rank 0's draw
            import torch.distributed as dist
            dist.broadcast(nxt, src=0, group=self.tp.group)
        return (full if return_logits else None), nxt

    def gather_logits(self, logits: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits (all-gathered over the vocab shards under TP)."""
        if self.tp is None:
            return logits
        import torch.distributed as dist
        parts = [torch.empty_like(logits) for _ in range(self.tp.world)]
        dist.all_gather(parts, logits.contiguous(), group=self.tp.group)
        return torch.cat(parts, dim=-1)[:, :self.vocab_size]

    def next_tokens(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy next token per row (int32); distributed over vocab shards under TP."""
        idx = self.argmax(logits)
        if self.tp is None:
            return idx
        from .tensor_parallel import distributed_argmax
        vals = logits.gather(1, idx.to(torch.int64).unsqueeze(1)).squeeze(1).float()
        return distributed_argmax(vals, idx, self.vocab_offset, self.tp).to(torch.int32)

    def argmax(self, logits: torch.Tensor) -> torch.Tensor:
        """int(logits[row].argmax()) for every row, on the device."""
        M, V = logits.shape
        out = torch.empty(M, dtype=torch.int32, device=logits.device)
        _lib.check(_lib.load().ps_argmax(out.data_ptr(), logits.data_ptr(), M, V, logits.stride(0),
                                         _lib.dtype_code(logits.dtype), _lib.stream_ptr(logits.device)), "argmax")
        return out


class StepGraph:
    """CUDA-graph replay of one ``forward_batch`` shape (the graph-capturable
    decode the reference's engine/cuda_graphs.py:17-26 asks for: block tables
    and start positions live in device buffers refreshed by copies, so one
    captured graph serves every step of the same batch shape).

    Fixed at capture: the chunk lengths ``q_lens``, ``max_blocks`` (table
    width) and ``max_ctx`` (upper bound on any sequence's context). Varying
    per replay: token ids, start positions, block tables.
    """

    def __init__(self, model: PagedCausalLM, q_lens: list[int], max_blocks: int, max_ctx: int,
                 start_pos: list[int], block_tables: list[list[int]], input_ids=None):
        self.m = model
        self.q_lens = list(q_lens)
        self.B = len(q_lens)
        self.T = int(sum(q_lens))
        self.max_blocks = max_blocks
        self.max_ctx = max_ctx
        dev = model.device
        buf, B, mb, ctx = pack_metadata(q_lens, start_pos, block_tables, model.block_size, model.num_blocks,
                                        max_blocks)
        self.meta_dev = torch.from_numpy(buf).to(dev)
        self.meta_host = torch.empty(buf.shape, dtype=torch.int32, pin_memory=True)
        self.ids_dev = torch.zeros(self.T, dtype=torch.int64, device=dev)
        self.ids_host = torch.empty(self.T, dtype=torch.int64, pin_memory=True)
        self.tok_host = torch.empty(self.B, dtype=torch.int32, pin_memory=True)
        if input_ids is not None:
            self.ids_dev.copy_(torch.as_tensor(np.asarray(input_ids, np.int64)))
        Bn = self.B
        self.meta = StepMeta(self.meta_dev[2 * Bn + 1:].view(Bn, mb), self.meta_dev[:Bn + 1],
                             self.meta_dev[Bn + 1:2 * Bn + 1], self.q_lens, [max_ctx] * Bn)
        self.last = (self.meta_dev[1:Bn + 1].to(torch.int64) - 1)
        self.launches_per_replay = 0
        self.graph = None
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up: sizes the workspaces, loads kernels
                self._body()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        before = _lib.launch_count()
        with torch.cuda.graph(self.graph):
            self.logits, self.tokens = self._body()
        self.launches_per_replay = _lib.launch_count() - before

    def _body(self):
        last = self.meta_dev[1:self.B + 1].to(torch.int64) - 1
        logits = self.m._forward(self.ids_dev, self.meta, last)
        return logits, self.m.next_tokens(logits)

    def release(self) -> None:
        """Drop the captured graph (before destroy_process_group when it
        holds NCCL calls)."""
        if self.graph is not None:
            self.graph.reset()
            self.graph = None

    def replay(self) -> None:
        """Re-run the captured step on the current device buffers."""
        self.graph.replay()

    def set_inputs(self, input_ids, start_pos: list[int], block_tables: list[list[int]]) -> None:
        """Host inputs -> pinned staging -> device buffers (async copies on
        the current stream). Validates like forward_batch."""
        buf, B, mb, ctx = pack_metadata(self.q_lens, start_pos, block_tables, self.m.block_size, self.m.num_blocks,
                                        self.max_blocks)
        if max(ctx) > self.max_ctx:
            raise IndexError(f"context {max(ctx)} exceeds the captured bound {self.max_ctx}")
        self.meta_host.numpy()[:] = buf
        self.ids_host.numpy()[:] = np.asarray(input_ids, np.int64).reshape(-1)
        self.meta_dev.copy_(self.meta_host, non_blocking=True)
        self.ids_dev.copy_(self.ids_host, non_blocking=True)

    def run(self, input_ids, start_pos: list[int], block_tables: list[list[int]]) -> np.ndarray:
        """One step end to end: host inputs in, host next-token ids out."""
        self.set_inputs(input_ids, start_pos, block_tables)
        self.graph.replay()
        self.tok_host.copy_(self.tokens, non_blocking=True)
        torch.cuda.current_stream(self.m.device).synchronize()
        return self.tok_host.numpy().copy()

    @property
    def h2d_bytes(self) -> int:
        return self.meta_host.numel() * 4 + self.ids_host.numel() * 8

    @property
    def d2h_bytes(self) -> int:
        return self.tok_host.numel() * 4
