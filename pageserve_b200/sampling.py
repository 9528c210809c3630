"""On-device next-token selection and its asynchronous host copy.

The reference reads every sequence's full logits row on the host and calls
``int(logits[-1].argmax())`` (server.py:47-51, engine/runner.py:79-83): one
device->host sync per sequence. Here the selection runs on the device for the
whole batch — greedy (``PagedCausalLM.argmax``), top-k, or sampling from the
top-k — and only the token ids cross to the host, through pinned memory with
an event, so the host can prepare the next step meanwhile.
"""

from __future__ import annotations

import torch

from . import _lib


def top_k(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(values float32 (M, k), indices int32 (M, k)) of each row of a 2-D
    logits tensor, sorted by value descending, ties by lowest index."""
    _lib.require_cuda(logits)
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("top_k: logits must be 2-D with contiguous rows")
    M, V = logits.shape
    vals = torch.empty((M, k), dtype=torch.float32, device=logits.device)
    idx = torch.empty((M, k), dtype=torch.int32, device=logits.device)
    _lib.check(_lib.load().ps_topk(vals.data_ptr(), idx.data_ptr(), logits.data_ptr(), M, V, logits.stride(0), k,
                                   _lib.dtype_code(logits.dtype), _lib.stream_ptr(logits.device)), "topk")
    return vals, idx


def sample_top_k(logits: torch.Tensor, k: int, temperature: float = 1.0, uniforms: torch.Tensor | None = None,
                 generator: torch.Generator | None = None) -> torch.Tensor:
    """One token per row sampled from softmax(top-k logits / temperature)
    by inverse CDF with one uniform per row (``uniforms``, float32 (M,), or
    drawn on the device from ``generator``). int32 (M,)."""
    vals, idx = top_k(logits, k)
    M = logits.shape[0]
    if uniforms is None:
        uniforms = torch.rand(M, device=logits.device, generator=generator, dtype=torch.float32)
    uniforms = uniforms.to(device=logits.device, dtype=torch.float32).contiguous()
    out = torch.empty(M, dtype=torch.int32, device=logits.device)
    _lib.check(_lib.load().ps_sample_topk(out.data_ptr(), vals.data_ptr(), idx.data_ptr(), uniforms.data_ptr(), M, k,
                                          float(temperature), _lib.stream_ptr(logits.device)), "sample_topk")
    return out


class HostTokens:
    """Token ids copied to pinned host memory on the current stream without
    blocking it; ``wait()`` (or ``ready()``) tells when they have landed."""

    def __init__(self, tokens: torch.Tensor):
        self.host = torch.empty(tokens.shape, dtype=tokens.dtype, pin_memory=True)
        self.host.copy_(tokens, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record(torch.cuda.current_stream(tokens.device))

    def ready(self) -> bool:
        return self.event.query()

    def wait(self) -> list[int]:
        self.event.synchronize()
        return self.host.tolist()
