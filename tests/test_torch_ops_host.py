"""torch.ops.pageserve_b200 registration (§ drop-in boundary: TORCH_LIBRARY
ops over the extern "C" core), on CPU: every operator is registered, its
Meta function gives the output shapes for tracing, and a CPU tensor raises
(no CPU fallback)."""

import pytest
import torch

from pageserve_b200 import ops as ops_mod


@pytest.fixture(scope="module")
def ops():
    if not ops_mod.LIB_PATH.exists():
        pytest.skip("torch ops library not built")
    return ops_mod.load()


def test_every_operator_is_registered(ops):
    for name in ops_mod.OPS:
        assert hasattr(ops, name), name
        assert torch._C._dispatch_has_kernel_for_dispatch_key(f"pageserve_b200::{name}", "CUDA"), name


def test_meta_shapes(ops):
    m = torch.device("meta")
    x = torch.empty(7, 2048, device=m, dtype=torch.bfloat16)
    qt = torch.empty(16 * 32 * 8192, device=m, dtype=torch.int8)
    sc = torch.empty(2560, 1, device=m)
    assert ops.w8a16_linear(x, qt, sc, 2560).shape == (7, 2560)
    assert ops.linear_swiglu(x, qt, sc, 22016).shape == (7, 11008)
    assert ops.linear16(x, torch.empty(300, 2048, device=m, dtype=torch.bfloat16)).shape == (7, 300)
    assert ops.rms_norm(x, torch.empty(2048, device=m, dtype=torch.bfloat16), 1e-6).shape == (7, 2048)
    y, s = ops.add_rms_norm(x, x, torch.empty(2048, device=m, dtype=torch.bfloat16), 1e-6)
    assert y.shape == s.shape == (7, 2048)
    q = torch.empty(9, 16, 128, device=m, dtype=torch.bfloat16)
    kc = torch.empty(10, 16, 2, 128, device=m, dtype=torch.bfloat16)
    i32 = dict(device=m, dtype=torch.int32)
    out = ops.paged_attention(q, kc, kc, torch.empty(2, 5, **i32), torch.empty(3, **i32), torch.empty(2, **i32), 8, 70)
    assert out.shape == q.shape and out.dtype == q.dtype
    v, i = ops.topk(torch.empty(4, 1000, device=m), 50)
    assert v.shape == i.shape == (4, 50) and i.dtype == torch.int32
    assert ops.argmax(torch.empty(4, 1000, device=m)).shape == (4,)
    qq, ss = ops.quantize_per_channel(torch.empty(64, 96, device=m))
    assert qq.shape == (64, 96) and qq.dtype == torch.int8 and ss.shape == (64, 1)


def test_cpu_tensors_raise(ops):
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        ops.rms_norm(x, torch.ones(64, dtype=torch.bfloat16), 1e-6)
