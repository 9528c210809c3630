"""On-device token selection (csrc/sampling.cu): top-k and top-k sampling
of logits rows, the batched replacement of the reference's per-sequence host
argmax (server.py:47-51, engine/runner.py:79-83).

* top_k equals a stable descending sort of each row (numpy, ties by lowest
  index), bit for bit, on bf16 rows of the 3B vocabulary width (many exact
  ties) and float32 rows; k = 1 equals the greedy argmax.
* sample_top_k picks, for the given uniforms, the inverse-CDF index of
  softmax(top-k / temperature) computed in float64 on the host (uniforms
  within 1e-5 of a CDF boundary are skipped: the device sums in float32).
* HostTokens lands the ids in pinned host memory behind an event."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _expected_topk(x: np.ndarray, k: int):
    order = np.lexsort((np.arange(x.shape[1])[None, :].repeat(x.shape[0], 0), -x), axis=1)[:, :k]
    return np.take_along_axis(x, order, 1), order


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("k", [1, 8, 50, 1024])
def test_topk_matches_stable_sort(dev, dtype, k):
    from pageserve_b200.sampling import top_k
    g = torch.Generator(device=dev)
    g.manual_seed(k)
    M, V = 65, 151936
    logits = (torch.randn(M, V, device=dev, generator=g) * 2).to(dtype)
    logits[3, 100] = logits[3, 7] = logits[3].max() + 1  # a tie at the top: lowest index first
    logits[4, :] = -float("inf")
    logits[4, 9] = 0.5
    vals, idx = top_k(logits, k)
    torch.cuda.synchronize()
    x = logits.float().cpu().numpy()
    ev, ei = _expected_topk(x, k)
    assert np.array_equal(idx.cpu().numpy(), ei)
    assert np.array_equal(vals.cpu().numpy(), ev)
    if k == 1:
        from pageserve_b200 import _lib
        out = torch.empty(M, dtype=torch.int32, device=dev)
        _lib.check(_lib.load().ps_argmax(out.data_ptr(), logits.data_ptr(), M, V, V, _lib.dtype_code(dtype),
                                         _lib.stream_ptr(dev)), "argmax")
        assert torch.equal(out, idx[:, 0])


def test_topk_rejects_bad_k(dev):
    from pageserve_b200.sampling import top_k
    x = torch.zeros(2, 100, device=dev, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        top_k(x, 101)
    with pytest.raises(Exception):
        top_k(x, 0)


@pytest.mark.parametrize("k,temp", [(1, 1.0), (8, 1.0), (50, 0.7), (40, 5.0)])
def test_sample_top_k_inverse_cdf(dev, k, temp):
    from pageserve_b200.sampling import HostTokens, sample_top_k, top_k
    g = torch.Generator(device=dev)
    g.manual_seed(100 + k)
    M, V = 64, 32000
    logits = (torch.randn(M, V, device=dev, generator=g) * 3).to(torch.bfloat16)
    u = torch.rand(M, device=dev, generator=g)
    toks = sample_top_k(logits, k, temp, uniforms=u)
    host = HostTokens(toks)
    got = host.wait()
    vals, idx = top_k(logits, k)
    v = vals.double().cpu().numpy()
    ix = idx.cpu().numpy()
    un = u.double().cpu().numpy()
    checked = 0
    for r in range(M):
        p = np.exp((v[r] - v[r, 0]) / temp)
        c = np.cumsum(p) / p.sum()
        if np.min(np.abs(c - un[r])) < 1e-5:
            continue
        j = int(np.searchsorted(c, un[r], side="right"))
        assert got[r] == ix[r, min(j, k - 1)], r
        checked += 1
    assert checked >= M - 2
    if k == 1:
        assert got == ix[:, 0].tolist()


def test_forward_batch_top_k_sampling(dev):
    """forward_batch(top_k=1) is the greedy pick; top_k sampling draws from
    the returned logits' top-k (same uniforms through sample_top_k)."""
    from pageserve_b200 import synthetic
    from pageserve_b200.model import PagedCausalLM
    from pageserve_b200.sampling import sample_top_k
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=2, perturb_norms_biases=True)
    m = PagedCausalLM.from_state_dict(sd, shape, device="cuda", dtype=torch.bfloat16, quantize=True)
    m.allocate_kv_cache(16, 4)
    ids = np.arange(10) % shape.vocab
    lg, greedy = m.forward_batch(ids, [6, 4], [0, 0], [[0, 1], [2]])
    _, k1 = m.forward_batch(ids, [6, 4], [0, 0], [[0, 1], [2]], top_k=1)
    assert torch.equal(greedy, k1)
    g1 = torch.Generator(device=dev).manual_seed(9)
    lg2, s1 = m.forward_batch(ids, [6, 4], [0, 0], [[0, 1], [2]], top_k=20, temperature=0.8, generator=g1)
    g2 = torch.Generator(device=dev).manual_seed(9)
    assert torch.equal(s1, sample_top_k(lg2, 20, 0.8, generator=g2))
