"""Tensor-parallel host logic on CPU: shard plans, and the column->row
protocol (sharded int8 weights keeping full-row scales, SUM all-reduce,
distributed argmax) over 2 gloo ranks — the structure of the reference's
tests/test_tensor_parallel.py, with the oracle doing the local math."""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import ops
from pageserve_b200 import synthetic
from pageserve_b200.tensor_parallel import ShardPlan, TPGroup, distributed_argmax


@pytest.mark.parametrize("shape", [synthetic.QWEN25_3B, synthetic.QWEN25_32B, synthetic.QWEN25_0_5B])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_partitions(shape, world):
    if shape.num_heads % world or shape.intermediate % world or \
            (shape.num_kv_heads < world and world % shape.num_kv_heads):
        with pytest.raises(AssertionError):
            ShardPlan(0, world, shape.num_heads, shape.num_kv_heads, shape.head_dim, shape.intermediate, shape.vocab)
        return
    plans = [ShardPlan(r, world, shape.num_heads, shape.num_kv_heads, shape.head_dim, shape.intermediate,
                       shape.vocab) for r in range(world)]
    group = shape.num_heads // shape.num_kv_heads
    assert sorted(h for p in plans for h in p.q_heads) == list(range(shape.num_heads))
    for p in plans:
        # every local q head reads a local kv head, with one local GQA group size
        assert all(h // group in p.kv_heads for h in p.q_heads)
        assert p.heads_local % p.kv_heads_local == 0
        for j, h in enumerate(p.q_heads):
            assert p.kv_heads[j // (p.heads_local // p.kv_heads_local)] == h // group
    kv_cover = sorted(set(h for p in plans for h in p.kv_heads))
    assert kv_cover == list(range(shape.num_kv_heads))
    assert sorted(c for p in plans for c in p.inter_cols) == list(range(shape.intermediate))
    assert sorted(v for p in plans for v in p.vocab_rows) == list(range(shape.vocab))


def _worker(rank, world, sync_file, data_file, result_file):
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"file://{sync_file}")
    d = torch.load(data_file, weights_only=True)
    tp = TPGroup(rank, world)
    x, w1, w2 = d["x"].numpy(), d["w1"].numpy(), d["w2"].numpy()
    s = w1.shape[0] // world
    # column-parallel (row slice of w1 quantizes identically)
    q1, s1 = ops.quantize_per_channel(w1[rank * s:(rank + 1) * s])
    h = ops.quantized_linear(x, q1, s1)
    # row-parallel: quantize the FULL w2, keep full-row scales, slice columns
    q2, s2 = ops.quantize_per_channel(w2)
    partial = torch.from_numpy(ops.quantized_linear(h, q2[:, rank * s:(rank + 1) * s], s2))
    out = tp.all_reduce_(partial.clone())
    # vocab-parallel argmax over the reduced rows, with a planted cross-rank tie
    logits = out.clone()
    logits[0, :] = 0.0
    logits[0, 3] = 5.0          # rank 0 owns column 3 of an 8-column split
    logits[0, 4 + 1] = 5.0      # rank 1 owns column 5: same value, larger index
    per = logits.shape[1] // world
    local = logits[:, rank * per:(rank + 1) * per]
    mx, idx = local.max(dim=1)
    tok = distributed_argmax(mx, idx, rank * per, tp)
    torch.save({"out": out, "tok": tok}, f"{result_file}.{rank}")
    dist.destroy_process_group()


def test_column_row_int8_protocol_matches_unsharded():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 16), dtype=np.float32)
    w1 = rng.standard_normal((8, 16), dtype=np.float32)
    w2 = rng.standard_normal((8, 8), dtype=np.float32)
    q1, s1 = ops.quantize_per_channel(w1)
    q2, s2 = ops.quantize_per_channel(w2)
    expected = ops.quantized_linear(ops.quantized_linear(x, q1, s1), q2, s2)
    with tempfile.TemporaryDirectory() as tmp:
        data = os.path.join(tmp, "d.pt")
        torch.save({"x": torch.from_numpy(x), "w1": torch.from_numpy(w1), "w2": torch.from_numpy(w2)}, data)
        mp.spawn(_worker, args=(2, os.path.join(tmp, "sync"), data, os.path.join(tmp, "r")), nprocs=2, join=True)
        r0 = torch.load(os.path.join(tmp, "r.0"), weights_only=True)
        r1 = torch.load(os.path.join(tmp, "r.1"), weights_only=True)
    assert torch.equal(r0["out"], r1["out"])  # every rank holds the identical reduced output
    np.testing.assert_allclose(r0["out"].numpy(), expected, atol=1e-4, rtol=1e-5)
    ref = r0["out"].clone()
    ref[0, :] = 0.0
    ref[0, 3] = 5.0
    ref[0, 5] = 5.0
    assert r0["tok"].tolist() == ref.argmax(dim=1).tolist() == r1["tok"].tolist()
    assert int(r0["tok"][0]) == 3  # first index wins across ranks
