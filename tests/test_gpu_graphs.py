"""CUDA-graph buckets (pageserve_b200/graphs.py; the per-batch-size decode
graphs of engine/cuda_graphs.py:13-26, 32-69, made replayable at new
positions). Steps of changing batch sizes and shapes — decode batches of 3, 5,
3 and 1 sequences (buckets 4, 8, 4, 1, with pad rows), a mixed decode +
prefill-chunk step twice — run through StepGraphs on one model and through
forward_batch on a second: tokens equal (near-ties allowed), logits within
1e-2, every real KV block equal, and one capture per bucket or shape."""

import numpy as np
import pytest
import torch

from pageserve_b200 import synthetic

pytestmark = pytest.mark.gpu


def test_step_graph_buckets_across_batch_shapes():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from pageserve_b200.graphs import StepGraphs
    from pageserve_b200.model import PagedCausalLM
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=33, perturb_norms_biases=True)
    bs, NB, pad_block = 4, 64, 63
    graph_m = PagedCausalLM.from_state_dict(sd, shape, device="cuda", dtype=torch.bfloat16, quantize=True)
    eager_m = PagedCausalLM.from_state_dict(sd, shape, device="cuda", dtype=torch.bfloat16, quantize=True)
    for m in (graph_m, eager_m):
        m.allocate_kv_cache(NB, bs)
    rng = np.random.default_rng(12)
    tables = [list(range(i * 10, i * 10 + 10)) for i in range(6)]  # blocks 0..59; 63 is the pad block
    lens = [9, 14, 5, 21, 2, 0]
    prompts = [rng.integers(0, shape.vocab, size=40) for _ in range(6)]
    hist = [i for i in range(6) if lens[i]]
    for m in (graph_m, eager_m):
        m.forward_batch(np.concatenate([prompts[i][:lens[i]] for i in hist]), [lens[i] for i in hist], [0] * len(hist),
                        [tables[i] for i in hist], return_logits=False)
    graphs = StepGraphs(graph_m, max_blocks=10, max_ctx=40, pad_block=pad_block)
    pos = {i: lens[i] for i in range(6)}
    steps = [([0, 1, 2], None), ([0, 1, 2, 3, 4], None), ([4, 2, 0], None), ([1, 3], (5, 7)), ([0, 2], (5, 6)),
             ([3], None)]
    for k, (dec, pre) in enumerate(steps):
        seqs = list(dec) + ([pre[0]] if pre else [])
        q_lens = [1] * len(dec) + ([pre[1]] if pre else [])
        starts = [pos[s] for s in seqs]
        ids = np.concatenate([prompts[s][p:p + q] for s, p, q in zip(seqs, starts, q_lens)])
        tabs = [tables[s] for s in seqs]
        got = graphs.run(ids, q_lens, starts, tabs)
        lg_g = graphs.logits(len(seqs), q_lens).float().cpu().numpy()
        lg_e, tok_e = eager_m.forward_batch(ids, q_lens, starts, tabs)
        lg_e = lg_e.float().cpu().numpy()
        err = float(np.abs(lg_g - lg_e).max() / np.abs(lg_e).max())
        assert err < 1e-2, (k, err)
        for i, (a, b) in enumerate(zip(got.tolist(), tok_e.cpu().tolist())):
            top = lg_e[i].max()
            assert a == b or top - lg_e[i, a] <= 2.0 ** -7 * abs(top), (k, i, a, b)
        for s, q in zip(seqs, q_lens):
            pos[s] += q
    # captures: decode buckets 4, 8, 1 and one mixed shape (the second mixed step has another chunk length)
    assert sorted(graphs.decode) == [1, 4, 8]
    assert len(graphs.mixed) == 2 and graphs.captures == 5
    torch.cuda.synchronize()
    real = [b for t in tables for b in t]
    kg, ke = graph_m.k_cache[:, real].float(), eager_m.k_cache[:, real].float()
    assert float((kg - ke).abs().max()) <= 2e-2 * float(ke.abs().max())
    graphs.release()
