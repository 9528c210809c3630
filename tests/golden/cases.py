"""Case definitions shared by the fixture generator and the tests.

Inputs are regenerated from per-case seeds (numpy PCG64, platform
independent), so the committed fixtures only need to hold the reference's
outputs.
"""

from __future__ import annotations

import random

import numpy as np

# name: (Hq, Hkv, D, block_size, num_blocks, chunks [(start_pos, T)], table_spec, seed)
# table_spec: ("perm", pool_seed) -> first ceil(total/bs) ids of a
# random.Random(pool_seed) shuffle of range(num_blocks); ("bump",) -> 0, 1, 2, ...
ATTENTION_CASES = {
    # tests/test_paged_attention.py:40-76 of the reference: full prefill at
    # an exact block boundary, a partial last block, a single token.
    "block_boundary": (8, 2, 16, 8, 10, [(0, 16)], ("perm", 1), 101),
    "partial_last_block": (8, 2, 16, 8, 10, [(0, 19)], ("perm", 2), 102),
    "single_token": (8, 2, 16, 8, 10, [(0, 1)], ("perm", 3), 103),
    # tests/test_paged_attention.py:99-140: prefill 9, then 3 decode steps.
    "prefill_then_decode": (8, 2, 16, 4, 20, [(0, 9), (9, 1), (10, 1), (11, 1)], ("bump",), 104),
    # Benchmark-configuration head shapes with chunked prefill and decode.
    "gqa8_d128_chunked": (16, 2, 128, 16, 64, [(0, 37), (37, 9), (46, 1), (47, 1)], ("perm", 7), 105),
    "gqa7_d64_decode": (14, 2, 64, 16, 32, [(0, 99), (99, 1), (100, 1)], ("perm", 11), 106),
    "gqa5_d128_long": (40, 8, 128, 16, 48, [(0, 40), (40, 700), (740, 1)], ("perm", 5), 107),
}

# Outputs of cases whose output has more rows than this are stored as the
# last rows plus whole-output sums.
FULL_OUTPUT_ROWS = 64
TAIL_ROWS = 8


def attention_case(name):
    Hq, Hkv, D, bs, NB, chunks, spec, seed = ATTENTION_CASES[name]
    total = max(s + t for s, t in chunks)
    nblk = (total + bs - 1) // bs
    if spec[0] == "perm":
        ids = list(range(NB))
        random.Random(spec[1]).shuffle(ids)
        table = ids[:nblk]
    else:
        table = list(range(nblk))
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((total, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((total, Hkv, D), dtype=np.float32)
    q = rng.standard_normal((total, Hq, D), dtype=np.float32)
    return dict(Hq=Hq, Hkv=Hkv, D=D, bs=bs, NB=NB, chunks=chunks, table=table, k=k, v=v, q=q, total=total)


def stores_full_output(name) -> bool:
    c = ATTENTION_CASES[name]
    return max(s + t for s, t in c[5]) <= FULL_OUTPUT_ROWS


def stores_cache(name) -> bool:
    Hq, Hkv, D, bs, NB = ATTENTION_CASES[name][:5]
    return NB * bs * Hkv * D <= 65536


CFG1_CTX = (37, 128, 255, 511)
CFG1_STRIDE = 37


def cfg1_inputs(vocab: int = 151936):
    """Token ids and block tables of BASELINE config 1: 4 sequences at
    context 37/128/255/511, block size 16, consecutive slices of a
    random.Random(0) permutation of a 256-block pool."""
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, vocab, size=c).astype(np.int64) for c in CFG1_CTX]
    ids = list(range(256))
    random.Random(0).shuffle(ids)
    tables, at = [], 0
    for c in CFG1_CTX:
        n = (c + 15) // 16
        tables.append(ids[at:at + n])
        at += n
    return prompts, tables


# Greedy decode fixtures (make_golden.make_greedy): name -> (shape, seed,
# perturb norms/biases, prompt lengths). "cfg1" is BASELINE config 1's model
# (Qwen2.5-0.5B shape, all 24 layers, HF init); "3b4" has the Qwen2.5-3B
# dimensions (hidden 2048, 16/2 heads, head_dim 128, intermediate 11008,
# vocab 151936) with 4 layers and randomised norms/biases.
GREEDY_STEPS = 32          # decode steps after the prefill (33 greedy decisions)
GREEDY_STRIDE = 149        # logits sample stride
GREEDY_POOL = 256          # KV pool blocks (block size 16)


def _greedy_cases():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent.parent))
    from pageserve_b200 import synthetic
    return {
        "cfg1": (synthetic.QWEN25_0_5B, 0, False, CFG1_CTX),
        "3b4": (synthetic.QWEN25_3B.with_layers(4), 1, True, (45, 300, 777, 1200)),
    }


GREEDY_CASES = _greedy_cases()


def greedy_inputs(name: str):
    """Prompts and block tables of a greedy fixture: seeded random token ids;
    each sequence's table is a consecutive slice of a random.Random(17)
    permutation of the GREEDY_POOL-block pool, long enough for prompt +
    GREEDY_STEPS + 1 tokens."""
    shape, seed, _, ctxs = GREEDY_CASES[name]
    rng = np.random.default_rng(1000 + seed)
    prompts = [rng.integers(0, shape.vocab, size=c).astype(np.int64) for c in ctxs]
    ids = list(range(GREEDY_POOL))
    random.Random(17).shuffle(ids)
    tables, at = [], 0
    for c in ctxs:
        n = (c + GREEDY_STEPS + 1 + 15) // 16
        tables.append(ids[at:at + n])
        at += n
    assert at <= GREEDY_POOL
    return prompts, tables


# Continuous-batching trace (make_golden.make_sched_trace): an 8-block pool of
# 4-token blocks, 3 sequences per step and 8 tokens per step over 5 requests,
# so prefill is chunked and the pool runs out (preemption + recompute).
SCHED_TRACE = {"num_blocks": 8, "block_size": 4, "max_batch_size": 3, "token_budget": 8,
               "prompt_lens": (5, 11, 3, 17, 8), "max_new": (6, 3, 9, 4, 5), "vocab": 512}


def sched_trace_prompts():
    rng = np.random.default_rng(404)
    return [rng.integers(0, SCHED_TRACE["vocab"], size=n).astype(np.int64) for n in SCHED_TRACE["prompt_lens"]]


def fake_next_token(input_ids, start_pos) -> int:
    """A deterministic stand-in for the model's greedy token."""
    return int((sum(int(t) for t in input_ids) * 31 + int(start_pos) * 7 + len(input_ids)) % SCHED_TRACE["vocab"])
