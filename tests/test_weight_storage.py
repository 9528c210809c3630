"""Host-side checks of the one-copy weight storage (CPU, no GPU needed): the
exact inverse of the kernels' 8 KB-block int8 layout, and the row views the
model hands out as its per-projection weights (engine/model.py:57-70
LayerWeights, engine/quantization.py:30-50 QuantizedWeight)."""

import numpy as np
import pytest
import torch

from pageserve_b200.quantization import QuantizedWeight, RowView, untile_int8_weight


def tile_ref(q: np.ndarray) -> np.ndarray:
    """The tiled layout, restated: [ceil(N/128)][ceil(K/64)][128][64], zero
    padded, 16-byte chunk c of row r stored at chunk slot c ^ ((r >> 1) & 3)."""
    N, K = q.shape
    nb, kt = (N + 127) // 128, (K + 63) // 64
    pad = np.zeros((nb * 128, kt * 64), np.int8)
    pad[:N, :K] = q
    blocks = pad.reshape(nb, 128, kt, 4, 16).transpose(0, 2, 1, 3, 4)
    out = np.empty_like(blocks)
    for r in range(128):
        for c in range(4):
            out[:, :, r, c ^ ((r >> 1) & 3)] = blocks[:, :, r, c]
    return out.reshape(-1)


@pytest.mark.parametrize("NK", [(128, 64), (136, 896), (300, 880), (2560, 2048), (7, 16), (513, 200)])
def test_untile_inverts_tiling(NK):
    rng = np.random.default_rng(NK[0] + NK[1])
    q = rng.integers(-127, 128, size=NK).astype(np.int8)
    back = untile_int8_weight(torch.from_numpy(tile_ref(q)), *NK)
    assert back.dtype == torch.int8 and tuple(back.shape) == NK
    assert np.array_equal(back.numpy(), q)


def _tiled_only(q: np.ndarray, scale: np.ndarray) -> QuantizedWeight:
    """A QuantizedWeight holding only the tiled copy, as the model keeps it."""
    w = QuantizedWeight.from_quantized(torch.from_numpy(q), torch.from_numpy(scale), torch.bfloat16)
    w._tiled = torch.from_numpy(tile_ref(q))
    w._q = None
    return w


def test_tiled_only_weight_reads_back():
    rng = np.random.default_rng(1)
    q = rng.integers(-127, 128, size=(300, 200)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=(300, 1)).astype(np.float32)
    w = _tiled_only(q, s)
    assert w.shape == (300, 200)
    assert w.storage_bytes == 300 * 200 + 300 * 4  # the reference's count (q + fp32 scales)
    assert np.array_equal(w.q.numpy(), q)
    assert torch.equal(w.get(), (torch.from_numpy(q).float() * torch.from_numpy(s)).to(torch.bfloat16))


def test_row_views_of_fused_weights():
    rng = np.random.default_rng(2)
    # q|k|v rows 256 + 128 + 128 (whole 128-row blocks) and a ragged split
    fused = rng.integers(-127, 128, size=(512, 320)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, size=(512, 1)).astype(np.float32)
    src = _tiled_only(fused, s)
    full_tiled = src.tiled()
    for rows in (slice(0, 256), slice(256, 384), slice(384, 512), slice(0, None, 2), slice(1, None, 2),
                 slice(100, 300)):
        v = RowView(src, rows, torch.bfloat16)
        assert v.shape == fused[rows].shape
        assert np.array_equal(v.q.numpy(), fused[rows])
        assert np.array_equal(v.scale.numpy(), s[rows])
        if rows.step is None and rows.start % 128 == 0:
            t = v.tiled()  # a view into the fused tiled copy, no new storage
            assert t.untyped_storage().data_ptr() == full_tiled.untyped_storage().data_ptr()
            assert np.array_equal(untile_int8_weight(t, *v.shape).numpy(), fused[rows])
