"""GPU parity of the CTA-pair W8A16 linear (tcgen05.mma.cta_group::2,
persistent, two TMEM accumulators; csrc/linear_tc2.cu) against the oracle.

The pair kernel is opt-in (PS_TC2=1: shapes with N a multiple of 256 and at
least one full round of 256 x BM tiles; PS_TC2=2: wherever legal); every
test here switches it on for its own calls. Cases: partial last token tiles
(the second CTA's half of the tile partly or wholly past M), more tiles than
resident pairs (several tiles per pair, so both accumulators and the ring
phases wrap), odd k-tile counts, bias + residual, SwiGLU, f16, and one tile
on one pair. engine/quantization.py:26-50 + F.linear and
engine/model.py:188-190 of the reference are the functions restated by the
oracle."""

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
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def pair_kernel_on(monkeypatch):
    monkeypatch.setenv("PS_TC2", "2")


def _t(a, dev, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)


def _round(x, dtype):
    return ops.round_bf16(x) if dtype == torch.bfloat16 else x.astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(96, 19456, 320), (200, 20480, 320), (129, 19456, 1024), (576, 22016, 2048),
                                   (128, 27648, 5120), (40, 256, 192), (300, 512, 448)])
def test_pair_linear_bias_residual(dev, M, N, K, dtype):
    from pageserve_b200.quantization import tile_int8_weight, w8a16_linear
    rng = np.random.default_rng(M * 31 + N + K)
    q = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=(N, 1)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    qd = torch.from_numpy(q).to(dev)
    y = w8a16_linear(_t(x, dev, dtype), qd, torch.from_numpy(scale).to(dev), _t(b, dev, dtype), _t(r, dev, dtype),
                     q_tiled=tile_int8_weight(qd))
    torch.cuda.synchronize()
    ref = ops.quantized_linear(_round(x, dtype), q, scale, _round(b, dtype)) + _round(r, dtype)
    assert rel_err(y.float().cpu().numpy(), ref) < REL_TOL


@pytest.mark.parametrize("M,I,K", [(129, 9728, 1024), (576, 11008, 2048), (300, 9728, 640)])
def test_pair_linear_swiglu(dev, M, I, K):
    from pageserve_b200.model import _interleave_rows
    from pageserve_b200.quantization import QuantizedWeight, linear_swiglu
    rng = np.random.default_rng(M + I)
    qg = rng.integers(-127, 128, size=(I, K)).astype(np.int8)
    qu = rng.integers(-127, 128, size=(I, K)).astype(np.int8)
    sg = rng.uniform(1e-3, 1e-2, size=(I, 1)).astype(np.float32)
    su = rng.uniform(1e-3, 1e-2, size=(I, 1)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32) * 0.5
    wg = QuantizedWeight.from_quantized(torch.from_numpy(qg).to(dev), torch.from_numpy(sg).to(dev), torch.bfloat16)
    wu = QuantizedWeight.from_quantized(torch.from_numpy(qu).to(dev), torch.from_numpy(su).to(dev), torch.bfloat16)
    y = linear_swiglu(_t(x, dev, torch.bfloat16), _interleave_rows(wg, wu, torch.bfloat16))
    torch.cuda.synchronize()
    g = ops.round_bf16(ops.quantized_linear(ops.round_bf16(x), qg, sg))
    u = ops.round_bf16(ops.quantized_linear(ops.round_bf16(x), qu, su))
    assert y.shape == (M, I)
    assert rel_err(y.float().cpu().numpy(), ops.silu(g) * u) < REL_TOL


def test_pair_linear_repeatable(dev):
    """Fixed accumulation order: two launches give identical bits, and the
    device status word stays clean (no barrier timed out)."""
    from pageserve_b200 import _lib
    from pageserve_b200.quantization import tile_int8_weight, w8a16_linear
    M, N, K = 576, 22016, 2048
    rng = np.random.default_rng(9)
    qd = torch.from_numpy(rng.integers(-127, 128, size=(N, K)).astype(np.int8)).to(dev)
    s = torch.from_numpy(rng.uniform(1e-3, 1e-2, size=(N, 1)).astype(np.float32)).to(dev)
    x = _t(rng.standard_normal((M, K), dtype=np.float32), dev, torch.bfloat16)
    qt = tile_int8_weight(qd)
    y1 = w8a16_linear(x, qd, s, q_tiled=qt)
    y2 = w8a16_linear(x, qd, s, q_tiled=qt)
    torch.cuda.synchronize()
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    _lib.raise_on_device_error()
