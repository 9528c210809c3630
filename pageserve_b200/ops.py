"""torch.ops.pageserve_b200.* — the hot-path operators registered with the
PyTorch dispatcher by libpageserve_torch_ops.so (torch_ops/pageserve_ops.cpp:
TORCH_LIBRARY over the extern "C" core). CUDA kernels plus Meta shape
functions, so the ops show up to torch tracing and dispatch; no CPU kernels
(a CPU tensor raises, there is no fallback).

    from pageserve_b200.ops import load
    ops = load()            # == torch.ops.pageserve_b200
    y = ops.rms_norm(x, w, 1e-6)
"""

from __future__ import annotations

from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpageserve_torch_ops.so"

OPS = ("write_kv", "paged_attention", "quantize_per_channel", "tile_int8_weight", "w8a16_linear", "linear16",
       "linear_swiglu", "rms_norm", "add_rms_norm", "apply_rope", "embedding", "argmax", "topk", "copy_kv_blocks")

_loaded = False


def load():
    """Register the operators (once) and return torch.ops.pageserve_b200."""
    global _loaded
    if not _loaded:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m pageserve_b200.build`")
        from . import _lib
        _lib.load()  # the C core first (the ops library links against it)
        torch.ops.load_library(str(LIB_PATH))
        _loaded = True
    return torch.ops.pageserve_b200
