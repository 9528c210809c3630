"""Seeded random-init Qwen2-family checkpoints for the benchmark and the tests.

No checkpoint can be downloaded on the machines this runs on, so the decoder
shapes named by the benchmark configurations (Qwen2.5-0.5B, -3B, -32B) are
instantiated with N(0, 0.02) weights, the same distribution HF's
``Qwen2PreTrainedModel._init_weights`` uses (``initializer_range=0.02``):
linears and embeddings N(0, 0.02), RMSNorm weights 1, q/k/v biases 0.
``perturb_norms_biases=True`` additionally randomises the norm weights and the
q/k/v biases so those code paths are exercised with non-trivial values.

Every tensor draws from its own ``numpy.random.default_rng([seed, index])``
stream, so any subset of layers can be regenerated bit-identically on any
machine (PCG64 + ziggurat are platform independent). State-dict keys follow
HF's Qwen2 naming, which is what the reference's loader reads
(engine/model.py:104-137).
"""

from __future__ import annotations

from dataclasses import dataclass, asdict, replace

import numpy as np


@dataclass(frozen=True)
class Qwen2Shape:
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6
    tie_embeddings: bool = True
    max_position: int = 32768

    def with_layers(self, n: int) -> "Qwen2Shape":
        return replace(self, num_layers=n)

    def to_dict(self) -> dict:
        return asdict(self)


# Shapes of the benchmark configurations (4, 5).
QWEN25_0_5B = Qwen2Shape(24, 896, 14, 2, 64, 4864, 151936, tie_embeddings=True)
QWEN25_3B = Qwen2Shape(36, 2048, 16, 2, 128, 11008, 151936, tie_embeddings=True)
QWEN25_32B = Qwen2Shape(64, 5120, 40, 8, 128, 27648, 152064, tie_embeddings=False)
# A tiny shape with the same structure, for fast fixture-level parity.
TINY = Qwen2Shape(2, 256, 4, 2, 64, 320, 512, rope_theta=1.0e4, tie_embeddings=False, max_position=256)

SHAPES = {"qwen2.5-0.5b": QWEN25_0_5B, "qwen2.5-3b": QWEN25_3B, "qwen2.5-32b": QWEN25_32B, "tiny": TINY}

_LAYER_TENSORS = (
    "input_layernorm.weight",
    "post_attention_layernorm.weight",
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.q_proj.bias",
    "self_attn.k_proj.bias",
    "self_attn.v_proj.bias",
    "self_attn.o_proj.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
)


def tensor_shapes(s: Qwen2Shape) -> dict[str, tuple[int, ...]]:
    """HF Qwen2 state-dict key -> shape, in a fixed order (the order fixes
    each tensor's RNG stream index)."""
    H, D = s.hidden, s.head_dim
    out: dict[str, tuple[int, ...]] = {"model.embed_tokens.weight": (s.vocab, H)}
    per_layer = {
        "input_layernorm.weight": (H,),
        "post_attention_layernorm.weight": (H,),
        "self_attn.q_proj.weight": (s.num_heads * D, H),
        "self_attn.k_proj.weight": (s.num_kv_heads * D, H),
        "self_attn.v_proj.weight": (s.num_kv_heads * D, H),
        "self_attn.q_proj.bias": (s.num_heads * D,),
        "self_attn.k_proj.bias": (s.num_kv_heads * D,),
        "self_attn.v_proj.bias": (s.num_kv_heads * D,),
        "self_attn.o_proj.weight": (H, s.num_heads * D),
        "mlp.gate_proj.weight": (s.intermediate, H),
        "mlp.up_proj.weight": (s.intermediate, H),
        "mlp.down_proj.weight": (H, s.intermediate),
    }
    for i in range(s.num_layers):
        for name in _LAYER_TENSORS:
            out[f"model.layers.{i}.{name}"] = per_layer[name]
    out["model.norm.weight"] = (H,)
    if not s.tie_embeddings:
        out["lm_head.weight"] = (s.vocab, H)
    return out


def _stream_index(key: str) -> int:
    """Stable stream id per key, independent of how many layers a shape has."""
    if key == "model.embed_tokens.weight":
        return 0
    if key == "model.norm.weight":
        return 1
    if key == "lm_head.weight":
        return 2
    parts = key.split(".")
    layer = int(parts[2])
    name = ".".join(parts[3:])
    return 16 + layer * 32 + _LAYER_TENSORS.index(name)


def generate_tensor(s: Qwen2Shape, key: str, seed: int, perturb_norms_biases: bool = False) -> np.ndarray:
    shape = tensor_shapes(s)[key]
    rng = np.random.default_rng([seed, _stream_index(key)])
    if key.endswith("layernorm.weight") or key == "model.norm.weight":
        if perturb_norms_biases:
            return (1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        return np.ones(shape, dtype=np.float32)
    if key.endswith(".bias"):
        if perturb_norms_biases:
            return (0.1 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        return np.zeros(shape, dtype=np.float32)
    w = rng.standard_normal(shape, dtype=np.float32)
    w *= np.float32(0.02)
    return w


def generate_state_dict(s: Qwen2Shape, seed: int = 0, perturb_norms_biases: bool = False) -> dict[str, np.ndarray]:
    """Full float32 state dict in HF Qwen2 key naming."""
    return {k: generate_tensor(s, k, seed, perturb_norms_biases) for k in tensor_shapes(s)}


class TorchStateDict:
    """Mapping view of a random-init state dict generated lazily on a torch
    device (N(0, 0.02) linears/embeddings, unit norms, zero biases): the fast
    path for benchmark-sized shapes (a 3B-shape model is generated on the GPU
    in well under a second per layer). The values come from torch's generator
    and differ from ``generate_state_dict``'s numpy streams; parity tests use
    the numpy streams."""

    def __init__(self, s: Qwen2Shape, seed: int = 0, device="cuda"):
        self.shape = s
        self.seed = seed
        self.device = device
        self._shapes = tensor_shapes(s)

    def __contains__(self, key) -> bool:
        return key in self._shapes

    def keys(self):
        return self._shapes.keys()

    def get(self, key, default=None):
        return self[key] if key in self._shapes else default

    def __getitem__(self, key):
        import torch

        shape = self._shapes[key]
        if key.endswith("layernorm.weight") or key == "model.norm.weight":
            return torch.ones(shape, dtype=torch.float32, device=self.device)
        if key.endswith(".bias"):
            return torch.zeros(shape, dtype=torch.float32, device=self.device)
        g = torch.Generator(device=self.device)
        g.manual_seed(self.seed * 1_000_003 + _stream_index(key))
        return torch.randn(shape, generator=g, dtype=torch.float32, device=self.device).mul_(0.02)
