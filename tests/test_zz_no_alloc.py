"""The allocation-free paged-attention entry point (ps_paged_attention_noalloc).

It exists for callers that cannot call cudaMalloc — e.g. a plugin whose host
serving engine owns all device memory through its own pool, or a latency-
critical path where cudaMalloc's implicit synchronisation is not allowed. It
keeps its split-context scratch in a static device array instead of a
caller-provided workspace. These tests call it through the C ABI and check it
against ps_paged_attention (the entry point with a workspace) on two
consecutive calls, plus the host-side rejection of batches whose scratch need
is above the static limit.

This file is named to be collected last, so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2  # the bf16 tolerance used by the other GPU tests
NOALLOC_LIMIT = 8 << 20  # PS_ATTN_NOALLOC_SCRATCH_BYTES in include/pageserve_b200.h


def rel_err(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _batch(seed, B, lo, hi, dev, Hq=16, Hkv=2, D=128, bs=16, q_lens=None):
    """B sequences at contexts U[lo, hi]; each sequence's queries are its last
    q_lens[b] positions (1 = a decode batch)."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(lo, hi + 1, size=B)
    ql = np.ones(B, np.int64) if q_lens is None else np.asarray(q_lens, np.int64)
    nblk = [(int(c) + bs - 1) // bs for c in ctx]
    NB = sum(nblk) + 5
    perm = rng.permutation(NB)
    mb = max(nblk)
    tab = np.full((B, mb), -1, np.int32)
    at = 0
    for b, n in enumerate(nblk):
        tab[b, :n] = perm[at:at + n]
        at += n
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    kc = torch.randn(NB, bs, Hkv, D, device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(NB, bs, Hkv, D, device=dev, generator=g, dtype=torch.bfloat16)
    total = int(ql.sum())
    q = torch.randn(total, Hq, D, device=dev, generator=g, dtype=torch.bfloat16)
    cu = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
    return dict(q=q, kc=kc, vc=vc, tab=torch.from_numpy(tab).to(dev), cu=torch.from_numpy(cu).to(dev),
                sp=torch.from_numpy((ctx - ql).astype(np.int32)).to(dev), B=B, total=total, max_q=int(ql.max()),
                mb=mb, max_ctx=int(ctx.max()), NB=NB, bs=bs, Hq=Hq, Hkv=Hkv, D=D)


def _args(c, out):
    return (out.data_ptr(), c["q"].data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["tab"].data_ptr(), c["mb"],
            c["cu"].data_ptr(), c["sp"].data_ptr(), c["B"], c["total"], c["max_q"], c["max_ctx"], c["NB"], c["bs"],
            c["Hq"], c["Hkv"], c["D"])


def _compare(c, call):
    """ps_paged_attention (caller workspace, unbounded split plan) against
    ps_paged_attention_noalloc on the same batch."""
    from pageserve_b200 import _lib
    lib = _lib.load()
    dev = c["q"].device
    stream = _lib.stream_ptr(dev)
    ws_bytes = lib.ps_paged_attention_workspace_size(c["B"], c["max_q"], c["max_ctx"], c["Hq"], c["Hkv"], c["D"])
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    ref = torch.empty_like(c["q"])
    got = torch.full_like(c["q"], float("nan"))
    _lib.check(lib.ps_paged_attention(*_args(c, ref), _lib.PS_BF16, ws.data_ptr(), ws_bytes, stream),
               "paged_attention")
    rc = lib.ps_paged_attention_noalloc(*_args(c, got), _lib.PS_BF16, stream)
    assert rc == _lib.PS_OK, _lib.last_error()
    torch.cuda.synchronize()
    assert torch.isfinite(got).all(), f"call {call}: unwritten output"
    assert rel_err(got.float(), ref.float()) < REL_TOL, f"call {call}"
    return ws_bytes


def test_noalloc_attention_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from pageserve_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = _lib.stream_ptr(dev)
    for call, (seed, B, lo, hi) in enumerate([(1, 16, 600, 2048), (2, 24, 300, 3000)]):
        c = _batch(seed, B, lo, hi, dev)
        ws_bytes = lib.ps_paged_attention_workspace_size(B, 1, c["max_ctx"], c["Hq"], c["Hkv"], c["D"])
        assert 0 < ws_bytes <= NOALLOC_LIMIT, "the case must use split scratch"
        _compare(c, call)
    del stream


def test_noalloc_prefill_batches_twice():
    """Prefill batches through the allocation-free entry point, each run twice
    in a row (the static scratch keeps the previous call's partials):
    * 40/8 heads (GQA group 5, the 32B shape's) at head_dim 128: the
      mma.sync prefill kernel with a split key range, whose unbounded split
      plan needs more than the static scratch, so the entry point shrinks it;
    * 16/2 heads at head_dim 128: the tcgen05 prefill kernel (no scratch);
    * a ragged mix of chunk lengths at head_dim 64 (14/2 heads)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    cases_ = [
        dict(seed=5, B=2, lo=900, hi=1400, Hq=40, Hkv=8, D=128, q_lens=[64, 64]),
        dict(seed=6, B=3, lo=200, hi=700, Hq=16, Hkv=2, D=128, q_lens=[128, 40, 97]),
        dict(seed=7, B=5, lo=300, hi=2000, Hq=14, Hkv=2, D=64, q_lens=[33, 1, 120, 7, 64]),
    ]
    for k, kw in enumerate(cases_):
        c = _batch(kw.pop("seed"), kw.pop("B"), kw.pop("lo"), kw.pop("hi"), dev, **kw)
        for call in range(2):
            ws_bytes = _compare(c, (k, call))
            if k == 0:
                assert ws_bytes > NOALLOC_LIMIT, "case 0 must need more split scratch than the static array holds"


def test_noalloc_decode_head_dim_64_twice():
    """Decode batch at head_dim 64 (14/2 heads, BASELINE config 1's shape):
    the cp.async decode kernel with split partials in the static scratch."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    c = _batch(9, 16, 500, 2500, dev, Hq=14, Hkv=2, D=64)
    for call in range(2):
        ws_bytes = _compare(c, call)
        assert 0 < ws_bytes <= NOALLOC_LIMIT


def test_noalloc_rejects_batches_above_the_static_scratch():
    from pageserve_b200 import _lib
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    lib = _lib.load()
    # A decode batch whose split partials exceed the static scratch: 275
    # sequences x 2 query tokens x 32 heads (8 per kv head) at head_dim 64.
    args = (275, 2, 4096, 32, 4, 64)  # seqs, max_q_len, max_ctx, q heads, kv heads, head_dim
    need = lib.ps_paged_attention_workspace_size(*args)
    assert need > NOALLOC_LIMIT
    fake = 1 << 20  # never dereferenced: the size check runs before any device access
    seqs, qlen, ctx, hq, hkv, d = args
    rc = lib.ps_paged_attention_noalloc(fake, fake, fake, fake, fake, 256, fake, fake, seqs, seqs * qlen, qlen, ctx,
                                        4096, 16, hq, hkv, d, _lib.PS_BF16, None)
    assert rc == _lib.PS_ERR_INVALID
    assert "static limit" in _lib.last_error()
