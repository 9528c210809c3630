"""torch.ops.pageserve_b200.* on the GPU: each registered operator runs the
same kernel as the ctypes path of the same function, so the results are
equal bit for bit (write_kv, paged attention, quantization + tiling, the W8A16
and 16-bit linears, SwiGLU linear, RMSNorm (+ residual), RoPE, embedding,
argmax, top-k, KV block copies), and the ops work inside a CUDA graph."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from pageserve_b200 import ops as ops_mod
    return ops_mod.load()


def test_torch_ops_equal_ctypes_path(ops):
    from pageserve_b200 import model as pm
    from pageserve_b200 import paged_attention as pa
    from pageserve_b200 import prefix, sampling
    from pageserve_b200.quantization import QuantizedWeight, linear16, linear_swiglu, quantize_per_channel
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    bf = torch.bfloat16
    # quantization, tiling, W8A16 linear (+bias, +residual), SwiGLU linear, 16-bit linear
    w = torch.randn(384, 256, device=dev, generator=g) * 0.05
    q1, s1 = ops.quantize_per_channel(w)
    q2, s2 = quantize_per_channel(w)
    assert torch.equal(q1, q2) and torch.equal(s1, s2)
    qw = QuantizedWeight.from_quantized(q2, s2, bf)
    t = ops.tile_int8_weight(q2)
    assert torch.equal(t, qw.tiled())
    x = torch.randn(37, 256, device=dev, generator=g).to(bf)
    b = torch.randn(384, device=dev, generator=g).to(bf)
    r = torch.randn(37, 384, device=dev, generator=g).to(bf)
    assert torch.equal(ops.w8a16_linear(x, t, s2, 384, b, r), qw.linear(x, b, r))
    assert torch.equal(ops.linear_swiglu(x, t, s2, 384), linear_swiglu(x, qw))
    wb = w.to(bf)
    assert torch.equal(ops.linear16(x, wb), linear16(x, wb))
    # norms, RoPE, embedding
    nw = torch.randn(256, device=dev, generator=g).to(bf)
    assert torch.equal(ops.rms_norm(x, nw, 1e-6), pm.rms_norm(x, nw, 1e-6))
    y1, s_1 = ops.add_rms_norm(x, x, nw, 1e-6)
    xr = torch.empty_like(x)
    y2 = pm.rms_norm_fused(x, nw, 1e-6, residual=x, residual_out=xr)
    assert torch.equal(y1, y2) and torch.equal(s_1, xr)
    cos, sin = pm.build_rope_cache(64, 64, 1e4, dev, bf)
    xq = torch.randn(9, 4, 64, device=dev, generator=g).to(bf)
    assert torch.equal(ops.apply_rope(xq, cos[3:12], sin[3:12]), pm.apply_rope(xq, cos[3:12], sin[3:12]))
    table = torch.randn(500, 256, device=dev, generator=g).to(bf)
    ids = torch.tensor([3, 499, 0, 17], device=dev)
    assert torch.equal(ops.embedding(ids, table), table[ids])
    # KV writes, paged attention, block copies
    kc = torch.zeros(20, 16, 2, 128, device=dev, dtype=bf)
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    k = torch.randn(40, 2, 128, device=dev, generator=g).to(bf)
    v = torch.randn(40, 2, 128, device=dev, generator=g).to(bf)
    tab = [5, 2, 9]
    ops.write_kv(kc, vc, torch.tensor(tab, dtype=torch.int32, device=dev), 16, 0, k, v)
    pa.write_kv(kc2, vc2, tab, 16, 0, k, v)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    qa = torch.randn(8, 16, 128, device=dev, generator=g).to(bf)
    bt = torch.tensor([tab], dtype=torch.int32, device=dev)
    cu = torch.tensor([0, 8], dtype=torch.int32, device=dev)
    sp = torch.tensor([32], dtype=torch.int32, device=dev)
    assert torch.equal(ops.paged_attention(qa, kc, vc, bt, cu, sp, 8, 40),
                       pa.paged_attention(qa, kc, vc, bt, cu, sp, 8, 40))
    kl, vl = kc.unsqueeze(0).clone(), vc.unsqueeze(0).clone()
    ops.copy_kv_blocks(kl, vl, torch.tensor([[5, 11]], dtype=torch.int32, device=dev))
    prefix.copy_blocks(kc, vc, [(5, 11)])
    assert torch.equal(kl[0], kc) and torch.equal(vl[0], vc)
    # selection
    logits = torch.randn(5, 3000, device=dev, generator=g).to(bf)
    assert torch.equal(ops.argmax(logits), sampling.top_k(logits, 1)[1][:, 0])  # first index of the maximum
    v1, i1 = ops.topk(logits, 10)
    v2, i2 = sampling.top_k(logits, 10)
    assert torch.equal(v1, v2) and torch.equal(i1, i2)


def test_torch_ops_in_a_cuda_graph(ops):
    from pageserve_b200 import model as pm
    dev = torch.device("cuda", 0)
    x = torch.randn(64, 512, device=dev).to(torch.bfloat16)
    w = torch.ones(512, device=dev, dtype=torch.bfloat16)
    ops.rms_norm(x, w, 1e-6)  # warm up outside the capture
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = ops.rms_norm(x, w, 1e-6)
    x.copy_(torch.randn(64, 512, device=dev).to(torch.bfloat16))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, pm.rms_norm(x, w, 1e-6))
    np.testing.assert_array_equal(y.isfinite().cpu().numpy(), True)
