"""Megatron tensor parallelism for the decode step (engine/tensor_parallel.py).

Reference-compatible primitives:
  ``column_parallel_linear(x, full_weight, rank, world_size)``  (tensor_parallel.py:21-31)
  ``row_parallel_linear(x_shard, full_weight, rank, world_size)`` (tensor_parallel.py:34-48)
with the same argument meaning and AssertionError on an uneven split; the
local product runs on this package's linear kernels and the SUM all-reduce
on ``torch.distributed`` (NCCL between GPUs, gloo on CPU).

The model path (``ShardPlan`` + ``PagedCausalLM.from_state_dict(tp=...)``)
pre-shards the weights once at load instead of slicing the full weight on
every call (the reference slices per call, tensor_parallel.py:30, 45):
  * q|k|v columns by heads: rank r owns q heads [r*Hq/W, (r+1)*Hq/W) and the
    kv heads they read; when W > Hkv each kv head is replicated on the
    W/Hkv ranks whose q heads use it.
  * gate|up columns by intermediate channel; o_proj and down_proj rows
    (their input dimension) likewise, followed by the SUM all-reduce of the
    (tokens, hidden) partial output; the residual is added once, by rank 0.
  * lm_head by vocabulary rows; greedy next tokens by a distributed argmax.
Row-parallel int8 shards keep the full-row quantization scale, so the sum of
the ranks' partials equals the unsharded quantized linear exactly.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ShardPlan:
    """What rank ``rank`` of ``world`` owns for a Qwen2 shape (host logic)."""
    rank: int
    world: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int

    def __post_init__(self):
        assert self.num_heads % self.world == 0, "q heads must divide evenly across ranks"
        assert self.intermediate % self.world == 0, "intermediate size must divide evenly across ranks"
        if self.num_kv_heads >= self.world:
            assert self.num_kv_heads % self.world == 0, "kv heads must divide evenly across ranks"
        else:
            assert self.world % self.num_kv_heads == 0, "ranks must divide evenly over kv heads"

    @property
    def heads_local(self) -> int:
        return self.num_heads // self.world

    @property
    def q_heads(self) -> range:
        return range(self.rank * self.heads_local, (self.rank + 1) * self.heads_local)

    @property
    def kv_heads(self) -> range:
        """kv heads this rank reads (replicated when world > num_kv_heads)."""
        group = self.num_heads // self.num_kv_heads
        first = self.q_heads.start // group
        last = (self.q_heads.stop - 1) // group
        return range(first, last + 1)

    @property
    def kv_heads_local(self) -> int:
        return len(self.kv_heads)

    @property
    def inter_local(self) -> int:
        return self.intermediate // self.world

    @property
    def inter_cols(self) -> range:
        return range(self.rank * self.inter_local, (self.rank + 1) * self.inter_local)

    @property
    def vocab_rows(self) -> range:
        per = -(-self.vocab // self.world)
        return range(min(self.vocab, self.rank * per), min(self.vocab, (self.rank + 1) * per))

    def q_rows(self) -> list[int]:
        d = self.head_dim
        return [h * d + i for h in self.q_heads for i in range(d)]

    def kv_rows(self) -> list[int]:
        d = self.head_dim
        return [h * d + i for h in self.kv_heads for i in range(d)]


# ------------------------------------------------ reference primitives ----

def _local_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """The local product on this package's kernel (no CPU fallback)."""
    if not (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype):
        raise TypeError("pageserve_b200 TP linears take bf16/f16 CUDA tensors (no CPU fallback)")
    from .quantization import linear16
    return linear16(x, w.contiguous())


def column_parallel_linear(x: torch.Tensor, full_weight: torch.Tensor, rank: int, world_size: int) -> torch.Tensor:
    """engine/tensor_parallel.py:21-31: this rank's shard of the output,
    x @ W[r*s:(r+1)*s].T; no communication."""
    out_features = full_weight.shape[0]
    assert out_features % world_size == 0, "output dim must divide evenly across ranks"
    shard = out_features // world_size
    return _local_linear(x, full_weight[rank * shard:(rank + 1) * shard])


def row_parallel_linear(x_shard: torch.Tensor, full_weight: torch.Tensor, rank: int, world_size: int,
                        group=None) -> torch.Tensor:
    """engine/tensor_parallel.py:34-48: partial = x_shard @ W[:, shard].T,
    then SUM all-reduce so every rank holds the full output."""
    in_features = full_weight.shape[1]
    assert in_features % world_size == 0, "input dim must divide evenly across ranks"
    shard = in_features // world_size
    partial = _local_linear(x_shard, full_weight[:, rank * shard:(rank + 1) * shard])
    dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


# ------------------------------------------------------ model helpers ----

@dataclass
class TPGroup:
    """The process group a sharded model reduces over."""
    rank: int
    world: int
    group: object = None

    @classmethod
    def from_default(cls) -> "TPGroup":
        return cls(dist.get_rank(), dist.get_world_size(), None)

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t


def distributed_argmax(local_max: torch.Tensor, local_idx: torch.Tensor, vocab_offset: int,
                       tp: TPGroup) -> torch.Tensor:
    """Greedy token over a vocab-sharded lm_head: each rank has the maximum
    logit and its local index per row; the winner is the largest value, ties
    to the lowest global index (torch.argmax's first-index rule), since ranks
    own increasing vocabulary ranges."""
    gidx = local_idx.to(torch.int64) + vocab_offset
    if tp.world == 1:
        return gidx
    vals = [torch.empty_like(local_max) for _ in range(tp.world)]
    idxs = [torch.empty_like(gidx) for _ in range(tp.world)]
    dist.all_gather(vals, local_max.contiguous(), group=tp.group)
    dist.all_gather(idxs, gidx.contiguous(), group=tp.group)
    v = torch.stack(vals)  # (world, M)
    i = torch.stack(idxs)
    best = v.max(dim=0).values
    # among ranks reaching the maximum, the smallest global index
    cand = torch.where(v == best.unsqueeze(0), i, torch.full_like(i, torch.iinfo(torch.int64).max))
    return cand.min(dim=0).values
