"""BASELINE configurations 2 and 3 at their own sizes, against the oracle.

* Config 2 (paged decode attention microbench): 64 sequences, 16/2 heads,
  head_dim 128, block 16, contexts U[512, 4096], q/K/V N(0, 1) in bf16, block
  tables drawn from a randomly permuted 20,000-block pool. The whole batch
  in one call of the product path (``paged_attention``, the TMA decode kernel
  with device-balanced key chunks + combine), every sequence checked against
  the oracle's ``paged_causal_attention_incremental``
  (engine/paged_attention.py:117-132) on the same bf16-rounded inputs.
* Config 3 (W8A16 linear sweep) at M = 256 and 2048 on the four Qwen2.5-3B
  projection shapes (K x N = 2048 x 2560 q|k|v with bias, 2048 x 2048 o_proj
  with residual, 2048 x 22016 gate|up, 11008 x 2048 down_proj with
  residual): int8 U[-127, 127], scales U[1e-3, 1e-2], x N(0, 1); through
  ``QuantizedWeight.linear`` (the model's tiled-weight path) against the
  oracle's ``quantized_linear`` (engine/quantization.py:26-50 +
  engine/model.py:25-26). gate|up is also run as the fused SwiGLU linear.

Tolerance: 2e-2 max relative error (bf16 results against float32)."""

import numpy as np
import pytest
import torch

from oracle import ops

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from pageserve_b200 import _lib
    _lib.load()
    d = torch.device("cuda", 0)
    _lib.ensure_status_word(d)
    return d


def test_config2_decode_attention_full_size(dev):
    from pageserve_b200 import _lib
    from pageserve_b200.paged_attention import paged_attention
    B, Hq, Hkv, D, bs, NB = 64, 16, 2, 128, 16, 20000
    rng = np.random.default_rng(0)
    ctx = rng.integers(512, 4096 + 1, size=B)
    nblk = [(int(c) + bs - 1) // bs for c in ctx]
    perm = rng.permutation(NB)
    mb = max(nblk)
    tab = np.full((B, mb), -1, np.int32)
    tables, at = [], 0
    for b, n in enumerate(nblk):
        tables.append(perm[at:at + n].tolist())
        tab[b, :n] = tables[-1]
        at += n
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    kc = torch.randn(NB, bs, Hkv, D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(NB, bs, Hkv, D, device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, D, device=dev, generator=g).to(torch.bfloat16)
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    sp = torch.from_numpy((ctx - 1).astype(np.int32)).to(dev)
    out = paged_attention(q, kc, vc, torch.from_numpy(tab).to(dev), cu, sp, 1, int(ctx.max()))
    torch.cuda.synchronize()
    _lib.raise_on_device_error()
    out = out.float().cpu().numpy()
    kcf, vcf, qf = kc.float().cpu().numpy(), vc.float().cpu().numpy(), q.float().cpu().numpy()
    worst = 0.0
    for b in range(B):
        ref = ops.paged_causal_attention_incremental(qf[b:b + 1], kcf, vcf, tables[b], bs, int(ctx[b]) - 1)
        e = rel_err(out[b:b + 1], ref)
        worst = max(worst, e)
        assert e < REL_TOL, f"seq {b} ctx {ctx[b]}: {e}"
    print(f"config 2: worst per-sequence rel err {worst:.2e} over {B} sequences, ctx {ctx.min()}..{ctx.max()}")


CFG3_SHAPES = {  # name: (N, K, epilogue)
    "qkv": (2560, 2048, "bias"),
    "o_proj": (2048, 2048, "residual"),
    "gate_up": (22016, 2048, "plain"),
    "down_proj": (2048, 11008, "residual"),
}


@pytest.mark.parametrize("M", [256, 2048])
@pytest.mark.parametrize("name", list(CFG3_SHAPES))
def test_config3_w8a16_linear_large_m(dev, name, M):
    from pageserve_b200.quantization import QuantizedWeight
    N, K, epi = CFG3_SHAPES[name]
    rng = np.random.default_rng(M + N + K)
    q = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=(N, 1)).astype(np.float32)
    x = ops.round_bf16(rng.standard_normal((M, K), dtype=np.float32))
    w = QuantizedWeight.from_quantized(torch.from_numpy(q).to(dev), torch.from_numpy(scale).to(dev), torch.bfloat16)
    w.release_row_major()  # the model's storage: the tiled copy only
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    bias = res = None
    ref = ops.quantized_linear(x, q, scale)
    if epi == "bias":
        b = ops.round_bf16(rng.standard_normal(N, dtype=np.float32))
        bias = torch.from_numpy(b).to(dev).to(torch.bfloat16)
        ref = ref + b
    elif epi == "residual":
        r = ops.round_bf16(rng.standard_normal((M, N), dtype=np.float32))
        res = torch.from_numpy(r).to(dev).to(torch.bfloat16)
        ref = ref + r
    y = w.linear(xb, bias, res)
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), ref) < REL_TOL


@pytest.mark.parametrize("M", [256, 2048])
def test_config3_gate_up_swiglu_large_m(dev, M):
    """The gate|up shape as the model runs it: one linear over the
    row-interleaved gate|up weight with silu(gate) * up in the epilogue."""
    from pageserve_b200.model import _interleave_rows
    from pageserve_b200.quantization import QuantizedWeight, linear_swiglu
    I, K = 11008, 2048
    rng = np.random.default_rng(M + 5)
    qg = rng.integers(-127, 128, size=(I, K)).astype(np.int8)
    qu = rng.integers(-127, 128, size=(I, K)).astype(np.int8)
    sg = rng.uniform(1e-3, 1e-2, size=(I, 1)).astype(np.float32)
    su = rng.uniform(1e-3, 1e-2, size=(I, 1)).astype(np.float32)
    x = ops.round_bf16(rng.standard_normal((M, K), dtype=np.float32) * 0.5)
    wg = QuantizedWeight.from_quantized(torch.from_numpy(qg).to(dev), torch.from_numpy(sg).to(dev), torch.bfloat16)
    wu = QuantizedWeight.from_quantized(torch.from_numpy(qu).to(dev), torch.from_numpy(su).to(dev), torch.bfloat16)
    w = _interleave_rows(wg, wu, torch.bfloat16)
    w.release_row_major()
    y = linear_swiglu(torch.from_numpy(x).to(dev).to(torch.bfloat16), w)
    torch.cuda.synchronize()
    gate = ops.round_bf16(ops.quantized_linear(x, qg, sg))
    up = ops.round_bf16(ops.quantized_linear(x, qu, su))
    assert rel_err(y.float().cpu().numpy(), ops.silu(gate) * up) < REL_TOL
