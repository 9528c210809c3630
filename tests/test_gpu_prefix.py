"""Prefix-cache-aware block sharing on the GPU (engine/prefix_cache.py:35-82:
sequences with a common prefix name the same physical blocks).

* ps_copy_kv_blocks copies whole blocks of every layer, bit-exact, and
  leaves every other block untouched.
* Two sequences whose block tables share the prefix's full blocks, one of
  them writing into a copy-on-write copy of the partly filled last block,
  decode together: their logits equal, bit for bit, those of the same two
  sequences on a second model where each owns a private copy of the prefix
  (same kernels, same cache contents), and the shared partial block keeps the
  parent's rows."""

import numpy as np
import pytest
import torch

from pageserve_b200 import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def test_copy_kv_blocks_bit_exact(dev):
    from pageserve_b200.prefix import copy_blocks
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    kc = torch.randn(3, 20, 16, 2, 128, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(3, 20, 16, 2, 128, device=dev, generator=g).to(torch.bfloat16)
    k0, v0 = kc.clone(), vc.clone()
    pairs = [(3, 7), (5, 0), (19, 2)]
    copy_blocks(kc, vc, pairs)
    torch.cuda.synchronize()
    ek, ev = k0.clone(), v0.clone()
    for s, d in pairs:
        ek[:, d] = k0[:, s]
        ev[:, d] = v0[:, s]
    assert torch.equal(kc, ek) and torch.equal(vc, ev)
    with pytest.raises(IndexError):
        copy_blocks(kc, vc, [(0, 20)])


def test_shared_prefix_blocks_with_copy_on_write(dev):
    from pageserve_b200.model import PagedCausalLM
    from pageserve_b200.prefix import fork
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=17, perturb_norms_biases=True)
    bs, NB = 4, 40
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, shape.vocab, size=14)  # 3 full blocks + 2 tokens
    kw = dict(device="cuda", dtype=torch.bfloat16, quantize=True)
    shared = PagedCausalLM.from_state_dict(sd, shape, **kw)
    private = PagedCausalLM.from_state_dict(sd, shape, **kw)
    for m in (shared, private):
        m.allocate_kv_cache(NB, bs)
    # shared model: A prefills, B forks A's table (3 shared blocks + a copy of the partial one)
    ta = [5, 17, 2, 30, 8, 9]
    shared.forward_batch(prompt, [14], [0], [ta], return_logits=False)
    free = iter([33, 34, 35, 36])
    tb = fork(shared, ta, 14, lambda: next(free))
    assert tb[:3] == ta[:3] and tb[3] == 33
    tb = tb + [next(free), next(free)]
    # private model: A and B each prefill the prompt into their own blocks
    pa, pb = [1, 3, 6, 10, 12, 13], [20, 21, 22, 23, 24, 25]
    for t in (pa, pb):  # one prefill per sequence, as the shared model's (same GEMM shapes, same bits)
        private.forward_batch(prompt, [14], [0], [t], return_logits=False)
    parent_rows = shared.k_cache[:, 30, :2].clone()
    for step, (xa, xb) in enumerate([(11, 200), (45, 45), (301, 7), (90, 91)]):
        pos = 14 + step
        lg_s, tok_s = shared.forward_batch([xa, xb], [1, 1], [pos, pos], [ta, tb])
        lg_p, tok_p = private.forward_batch([xa, xb], [1, 1], [pos, pos], [pa, pb])
        assert torch.equal(lg_s, lg_p), f"step {step}: shared-block logits differ from private copies"
        assert torch.equal(tok_s, tok_p)
    torch.cuda.synchronize()
    assert torch.equal(shared.k_cache[:, 30, :2], parent_rows), "the parent's partial block changed"
    # A's rows 14.. live in block 30 (slots 2, 3), B's in its copy 33
    assert torch.equal(shared.k_cache[:, 30, 2:], private.k_cache[:, 10, 2:])
    assert torch.equal(shared.k_cache[:, 33, 2:], private.k_cache[:, 23, 2:])
