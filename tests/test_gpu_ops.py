"""GPU parity of each hot-path operator against the oracle / the reference's
golden outputs (tolerance: 2e-2 max relative error for bf16 results against
float32, bit-exact for KV-slot writes and quantization)."""

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from oracle import ops

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
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


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16)


# ------------------------------------------------------------ write_kv ----

@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_write_kv_fp32_bit_exact_vs_reference(dev, name):
    from pageserve_b200.paged_attention import write_kv
    g = np.load(GOLDEN / "ops_paged_attention.npz")
    c = cases.attention_case(name)
    kc = torch.zeros((c["NB"], c["bs"], c["Hkv"], c["D"]), device=dev)
    vc = torch.zeros_like(kc)
    for s, t in c["chunks"]:
        write_kv(kc, vc, c["table"], c["bs"], s, torch.from_numpy(c["k"][s:s + t]).to(dev),
                 torch.from_numpy(c["v"][s:s + t]).to(dev))
    if cases.stores_cache(name):
        assert np.array_equal(kc.cpu().numpy(), g[f"{name}/k_cache"])
        assert np.array_equal(vc.cpu().numpy(), g[f"{name}/v_cache"])
    else:
        ko = np.zeros(kc.shape, np.float32)
        vo = np.zeros(vc.shape, np.float32)
        ops.write_kv(ko, vo, c["table"], c["bs"], 0, c["k"], c["v"])
        assert np.array_equal(kc.cpu().numpy(), ko)
        assert np.array_equal(vc.cpu().numpy(), vo)


def test_write_kv_bf16_bits_and_untouched_slots(dev):
    from pageserve_b200.paged_attention import write_kv
    rng = np.random.default_rng(5)
    NB, bs, Hkv, D = 40, 16, 2, 128
    table = list(rng.permutation(NB)[:9])
    k = rng.standard_normal((70, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((70, Hkv, D), dtype=np.float32)
    init = rng.standard_normal((NB, bs, Hkv, D), dtype=np.float32)
    kc = _bf16(init, dev)
    vc = _bf16(init, dev)
    write_kv(kc, vc, table, bs, 63, _bf16(k[:7], dev), _bf16(v[:7], dev))
    ko = ops.to_bf16_bits(init)
    vo = ko.copy()
    ops.write_kv(ko, vo, table, bs, 63, ops.to_bf16_bits(k[:7]), ops.to_bf16_bits(v[:7]))
    assert np.array_equal(kc.view(torch.int16).cpu().numpy().view(np.uint16), ko)
    assert np.array_equal(vc.view(torch.int16).cpu().numpy().view(np.uint16), vo)


def test_write_kv_short_table_raises_index_error(dev):
    from pageserve_b200.paged_attention import write_kv
    kc = torch.zeros((4, 16, 2, 64), device=dev, dtype=torch.bfloat16)
    k = torch.zeros((2, 2, 64), device=dev, dtype=torch.bfloat16)
    with pytest.raises(IndexError):
        write_kv(kc, kc.clone(), [0], 16, 15, k, k)


# ----------------------------------------------------------- attention ----

@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_paged_attention_matches_reference(dev, name, dtype):
    from pageserve_b200.paged_attention import paged_causal_attention_incremental, write_kv
    g = np.load(GOLDEN / "ops_paged_attention.npz")
    c = cases.attention_case(name)
    if c["D"] not in (64, 128):
        # head_dim 16 (the reference's tiny test shape): run the same case
        # padded to 64 with zeros — scores and outputs are unchanged.
        pad = 64 - c["D"]
        for key in ("k", "v", "q"):
            c[key] = np.concatenate([c[key], np.zeros((*c[key].shape[:2], pad), np.float32)], axis=-1)
        # the softmax scale uses the padded head_dim; rescale q to compensate
        c["q"] = c["q"] * np.float32(np.sqrt(64.0 / c["D"]))
        D = 64
    else:
        D = c["D"]
    kc = torch.zeros((c["NB"], c["bs"], c["Hkv"], D), device=dev, dtype=dtype)
    vc = torch.zeros_like(kc)
    outs = []
    for s, t in c["chunks"]:
        write_kv(kc, vc, c["table"], c["bs"], s, torch.from_numpy(c["k"][s:s + t]).to(dev, dtype),
                 torch.from_numpy(c["v"][s:s + t]).to(dev, dtype))
        o = paged_causal_attention_incremental(torch.from_numpy(c["q"][s:s + t]).to(dev, dtype), kc, vc, c["table"],
                                               c["bs"], s)
        outs.append(o.float().cpu().numpy()[..., :c["D"]])
    out = np.concatenate(outs, axis=0)
    if cases.stores_full_output(name):
        ref = g[f"{name}/out"]
        assert rel_err(out, ref) < REL_TOL
    else:
        assert rel_err(out[-cases.TAIL_ROWS:], g[f"{name}/out_tail"]) < REL_TOL
        sums = out.astype(np.float64).sum(axis=(1, 2))
        assert np.abs(sums - g[f"{name}/out_sum"]).max() < REL_TOL * np.abs(out).max() * out.shape[1] * out.shape[2]


@pytest.mark.parametrize("B,lo,hi", [(8, 512, 4096), (3, 1, 300), (64, 17, 700)])
def test_batched_decode_attention_split_context(dev, B, lo, hi):
    """Config-2 style batch (16/2 heads, D 128, bs 16, scrambled pool): the
    split-context decode kernel + combine against the oracle."""
    from pageserve_b200.paged_attention import paged_attention
    rng = np.random.default_rng(B)
    Hq, Hkv, D, bs = 16, 2, 128, 16
    ctx = rng.integers(lo, hi + 1, size=B)
    nblk = [(int(c) + bs - 1) // bs for c in ctx]
    NB = sum(nblk) + 7
    perm = rng.permutation(NB)
    tables, at = [], 0
    for n in nblk:
        tables.append(perm[at:at + n].tolist())
        at += n
    kc_np = rng.standard_normal((NB, bs, Hkv, D), dtype=np.float32)
    vc_np = rng.standard_normal((NB, bs, Hkv, D), dtype=np.float32)
    q_np = rng.standard_normal((B, Hq, D), dtype=np.float32)
    kc = _bf16(kc_np, dev)
    vc = _bf16(vc_np, dev)
    mb = max(nblk)
    tab = np.full((B, mb), -1, np.int32)
    for b, t in enumerate(tables):
        tab[b, :len(t)] = t
    cu = np.arange(B + 1, dtype=np.int32)
    sp = (ctx - 1).astype(np.int32)
    out = paged_attention(_bf16(q_np, dev), kc, vc, torch.from_numpy(tab).to(dev), torch.from_numpy(cu).to(dev),
                          torch.from_numpy(sp).to(dev), 1, int(ctx.max()))
    out = out.float().cpu().numpy()
    kcr = ops.round_bf16(kc_np)
    vcr = ops.round_bf16(vc_np)
    qr = ops.round_bf16(q_np)
    for b in range(B):
        ref = ops.paged_causal_attention_incremental(qr[b:b + 1], kcr, vcr, tables[b], bs, int(sp[b]))
        assert rel_err(out[b:b + 1], ref) < REL_TOL, f"seq {b} ctx {ctx[b]}"


def test_mixed_prefill_and_decode_runs(dev):
    """A chunked-prefill chunk at start_pos > 0 next to decode rows."""
    from pageserve_b200.paged_attention import paged_attention
    rng = np.random.default_rng(11)
    Hq, Hkv, D, bs = 16, 2, 128, 16
    NB = 128
    perm = rng.permutation(NB)
    kc_np = rng.standard_normal((NB, bs, Hkv, D), dtype=np.float32)
    vc_np = rng.standard_normal((NB, bs, Hkv, D), dtype=np.float32)
    # sequence 0: chunk of 40 tokens at start 300; sequence 1: chunk of 77 at 0
    specs = [(300, 40), (0, 77)]
    tables = [perm[:22].tolist(), perm[22:30].tolist()]
    q_np = rng.standard_normal((117, Hq, D), dtype=np.float32)
    tab = np.full((2, 22), -1, np.int32)
    for b, t in enumerate(tables):
        tab[b, :len(t)] = t
    cu = np.array([0, 40, 117], np.int32)
    sp = np.array([300, 0], np.int32)
    out = paged_attention(_bf16(q_np, dev), _bf16(kc_np, dev), _bf16(vc_np, dev), torch.from_numpy(tab).to(dev),
                          torch.from_numpy(cu).to(dev), torch.from_numpy(sp).to(dev), 77, 340).float().cpu().numpy()
    kcr, vcr, qr = ops.round_bf16(kc_np), ops.round_bf16(vc_np), ops.round_bf16(q_np)
    for b, (s, t) in enumerate(specs):
        ref = ops.paged_causal_attention_incremental(qr[cu[b]:cu[b + 1]], kcr, vcr, tables[b], bs, s)
        assert rel_err(out[cu[b]:cu[b + 1]], ref) < REL_TOL


# -------------------------------------------------------- quantization ----

def test_quantize_per_channel_bit_exact(dev):
    from pageserve_b200.quantization import QuantizedWeight, quantize_per_channel
    g = np.load(GOLDEN / "ops_quant.npz")
    q, s = quantize_per_channel(torch.from_numpy(g["w"]).to(dev))
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(s.cpu().numpy(), g["scale"])
    qw = QuantizedWeight(torch.from_numpy(g["w"]))  # CPU weight -> quantized on the GPU
    assert qw.storage_bytes == int(g["storage_bytes"])
    y = qw.linear(torch.from_numpy(g["x"]).to(dev), torch.from_numpy(g["b"]).to(dev))
    assert rel_err(y.cpu().numpy(), g["y"]) < 1e-5


# (96, 11008): few row groups and a long K, the small-M kernel's cp.async ring
# at M <= 8; (9480, 880) and (4808, 1040): ragged in N (not a multiple of 16)
# and K (not a multiple of 64), with 593 / 301 row groups
@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 64, 130])
@pytest.mark.parametrize("NK", [(2560, 2048), (2048, 2048), (96, 11008), (136, 896), (9480, 880), (4808, 1040)])
def test_w8a16_linear_matches_oracle(dev, M, NK):
    from pageserve_b200.quantization import w8a16_linear
    N, K = NK
    rng = np.random.default_rng(M * 7 + N)
    q = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=(N, 1)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    xb = _bf16(x, dev)
    y = w8a16_linear(xb, torch.from_numpy(q).to(dev), torch.from_numpy(scale).to(dev), _bf16(b, dev), _bf16(r, dev))
    ref = ops.quantized_linear(ops.round_bf16(x), q, scale, ops.round_bf16(b)) + ops.round_bf16(r)
    assert rel_err(y.float().cpu().numpy(), ref) < REL_TOL


def test_w8a16_linear_fp32_tight(dev):
    from pageserve_b200.quantization import w8a16_linear
    rng = np.random.default_rng(3)
    q = rng.integers(-127, 128, size=(64, 160)).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=(64, 1)).astype(np.float32)
    x = rng.standard_normal((5, 160), dtype=np.float32)
    y = w8a16_linear(torch.from_numpy(x).to(dev), torch.from_numpy(q).to(dev), torch.from_numpy(scale).to(dev))
    np.testing.assert_allclose(y.cpu().numpy(), ops.quantized_linear(x, q, scale), rtol=1e-5, atol=1e-5)


def test_linear16_lm_head(dev):
    from pageserve_b200.quantization import linear16
    rng = np.random.default_rng(9)
    w = rng.standard_normal((3000, 896), dtype=np.float32) * 0.02
    x = rng.standard_normal((4, 896), dtype=np.float32)
    y = linear16(_bf16(x, dev), _bf16(w, dev))
    assert rel_err(y.float().cpu().numpy(), ops.linear(ops.round_bf16(x), ops.round_bf16(w))) < REL_TOL


# ---------------------------------------------------------- norm / rope ----

def test_rms_norm_and_residual(dev):
    from pageserve_b200.model import rms_norm, rms_norm_fused
    g = np.load(GOLDEN / "ops_norm_rope.npz")
    y = rms_norm(torch.from_numpy(g["x"]).to(dev), torch.from_numpy(g["w"]).to(dev), 1e-6)
    np.testing.assert_allclose(y.cpu().numpy(), g["y"], rtol=1e-5, atol=1e-5)
    rng = np.random.default_rng(1)
    for H in (896, 2048, 5120):
        x = rng.standard_normal((7, H), dtype=np.float32)
        r = rng.standard_normal((7, H), dtype=np.float32)
        w = 1 + 0.1 * rng.standard_normal(H, dtype=np.float32)
        ro = torch.empty((7, H), device=dev, dtype=torch.bfloat16)
        y = rms_norm_fused(_bf16(x, dev), _bf16(w, dev), 1e-6, residual=_bf16(r, dev), residual_out=ro)
        s = ops.round_bf16(ops.round_bf16(x) + ops.round_bf16(r))
        assert np.array_equal(ro.float().cpu().numpy(), s)
        assert rel_err(y.float().cpu().numpy(), ops.rms_norm(s, ops.round_bf16(w), 1e-6)) < REL_TOL


def test_apply_rope_matches_reference(dev):
    from pageserve_b200.model import apply_rope
    g = np.load(GOLDEN / "ops_norm_rope.npz")
    sp = int(g["start_pos"])
    out = apply_rope(torch.from_numpy(g["q"]).to(dev), torch.from_numpy(g["cos"][sp:sp + 5]).to(dev),
                     torch.from_numpy(g["sin"][sp:sp + 5]).to(dev))
    np.testing.assert_allclose(out.cpu().numpy(), g["q_rope"], rtol=1e-5, atol=1e-5)


def test_fused_rope_qkv_write_kv(dev):
    from pageserve_b200 import _lib
    from pageserve_b200.model import build_rope_table_f32
    rng = np.random.default_rng(4)
    T, Hq, Hkv, D, bs, NB = 9, 16, 2, 128, 16, 12
    qkv = rng.standard_normal((T, (Hq + 2 * Hkv) * D), dtype=np.float32)
    table = [5, 2, 9]
    start = 27
    pos = np.arange(start, start + T, dtype=np.int32)
    slots = np.asarray([table[p // bs] * bs + p % bs for p in pos], np.int32)
    slots[3] = -1  # skipped write
    cos, sin = build_rope_table_f32(64, D, 1.0e6, dev)
    q_out = torch.empty((T, Hq, D), device=dev, dtype=torch.bfloat16)
    kc = torch.zeros((NB, bs, Hkv, D), device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qkv_d = _bf16(qkv, dev)
    pos_d = torch.from_numpy(pos).to(dev)      # keep the device buffers alive
    slots_d = torch.from_numpy(slots).to(dev)  # until the kernel has run
    _lib.check(_lib.load().ps_rope_qkv_write_kv(
        q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), qkv_d.data_ptr(), pos_d.data_ptr(), slots_d.data_ptr(),
        cos.data_ptr(), sin.data_ptr(), 64, T, Hq, Hkv, D, NB * bs, _lib.PS_BF16, _lib.stream_ptr()), "rope")
    torch.cuda.synchronize()
    ocos, osin = ops.build_rope_cache(64, D, 1.0e6)
    x = ops.round_bf16(qkv)
    qr = ops.apply_rope(x[:, :Hq * D].reshape(T, Hq, D), ocos[pos], osin[pos])
    kr = ops.apply_rope(x[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D), ocos[pos], osin[pos])
    vr = x[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    assert rel_err(q_out.float().cpu().numpy(), qr) < 1e-2
    kcn = kc.float().cpu().numpy().reshape(NB * bs, Hkv, D)
    vcn = vc.float().cpu().numpy().reshape(NB * bs, Hkv, D)
    written = set()
    for t in range(T):
        if slots[t] < 0:
            continue
        written.add(int(slots[t]))
        assert rel_err(kcn[slots[t]], kr[t]) < 1e-2
        assert np.array_equal(vcn[slots[t]], vr[t])  # v is a bit-exact copy
    untouched = [s for s in range(NB * bs) if s not in written]
    assert not np.any(kcn[untouched]) and not np.any(vcn[untouched])


def test_argmax_first_index(dev):
    from pageserve_b200.model import PagedCausalLM
    rng = np.random.default_rng(2)
    lg = rng.standard_normal((5, 151936), dtype=np.float32)
    lg[2, 100] = lg[2, 7] = 50.0  # tie: first index wins
    t = _bf16(lg, dev)
    out = PagedCausalLM.argmax(None, t).cpu().numpy()
    ref = ops.round_bf16(lg).argmax(-1)
    assert out.tolist() == ref.tolist()
    assert out[2] == 7


def test_embedding_out_of_range_sets_device_status(dev):
    from pageserve_b200 import _lib
    table = torch.randn(10, 64, device=dev, dtype=torch.bfloat16)
    ids = torch.tensor([1, 12, 3], device=dev, dtype=torch.int64)
    out = torch.empty(3, 64, device=dev, dtype=torch.bfloat16)
    _lib.device_status(clear=True)
    _lib.check(_lib.load().ps_embedding(out.data_ptr(), ids.data_ptr(), table.data_ptr(), 3, 64, 10,
                                        _lib.PS_BF16, _lib.stream_ptr()), "embedding")
    assert _lib.device_status(clear=True) == 3
    assert torch.equal(out[0], table[1]) and not out[1].any()


def _tile_ref(q):
    """numpy restatement of the 8 KB-block layout [N/128][K/64][128][64] with
    16-byte chunk c of row r stored in slot c ^ ((r >> 1) & 3)."""
    N, K = q.shape
    nb, kt = -(-N // 128), -(-K // 64)
    pad = np.zeros((nb * 128, kt * 64), np.int8)
    pad[:N, :K] = q
    blocks = pad.reshape(nb, 128, kt, 4, 16).transpose(0, 2, 1, 3, 4).copy()  # [nb][kt][r][c][16]
    out = np.empty_like(blocks)
    for r in range(128):
        for c in range(4):
            out[:, :, r, c ^ ((r >> 1) & 3)] = blocks[:, :, r, c]
    return out.reshape(-1)


@pytest.mark.parametrize("NK", [(136, 896), (300, 880), (2560, 2048)])
def test_tile_int8_weight_layout(dev, NK):
    from pageserve_b200.quantization import tile_int8_weight
    rng = np.random.default_rng(NK[0])
    q = rng.integers(-127, 128, size=NK).astype(np.int8)
    t = tile_int8_weight(torch.from_numpy(q).to(dev)).cpu().numpy()
    assert np.array_equal(t, _tile_ref(q))


@pytest.mark.parametrize("M", [1, 5, 16, 64, 130, 576])
@pytest.mark.parametrize("NK", [(2560, 2048), (136, 896), (300, 880), (2048, 11008), (9480, 880), (4808, 1040)])
def test_w8a16_linear_tiled_matches_oracle(dev, M, NK):
    from pageserve_b200.quantization import tile_int8_weight, w8a16_linear
    N, K = NK
    rng = np.random.default_rng(M * 13 + N)
    q = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=(N, 1)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    qd = torch.from_numpy(q).to(dev)
    y = w8a16_linear(_bf16(x, dev), qd, torch.from_numpy(scale).to(dev), _bf16(b, dev), _bf16(r, dev),
                     q_tiled=tile_int8_weight(qd))
    ref = ops.quantized_linear(ops.round_bf16(x), q, scale, ops.round_bf16(b)) + ops.round_bf16(r)
    assert rel_err(y.float().cpu().numpy(), ref) < REL_TOL


@pytest.mark.parametrize("MNK", [(576, 2560, 2048), (576, 2048, 11008), (130, 2048, 5504), (256, 300, 8192)])
def test_split_k_exchange_paths_agree(dev, MNK):
    """Split-K tiles reduce their partial sums through the caller's workspace
    (L2) or, without one, through the cluster's shared memories: both sum
    the splits in the same order, so the outputs are bit-identical, and both
    match the oracle."""
    import ctypes

    from pageserve_b200 import _lib
    from pageserve_b200.quantization import tile_int8_weight
    M, N, K = MNK
    lib = _lib.load()
    rng = np.random.default_rng(M + N + K)
    q = rng.integers(-127, 128, size=(N, K)).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=(N, 1)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    qt = tile_int8_weight(torch.from_numpy(q).to(dev))
    xd, rd = _bf16(x, dev), _bf16(r, dev)
    sd = torch.from_numpy(scale).to(dev)
    need = lib.ps_w8a16_linear_tiled_workspace_size(M, N, K)
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    outs = []
    for wsp, wsb in ((ws.data_ptr(), need), (None, 0)):
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        for _ in range(2):
            rc = lib.ps_w8a16_linear_tiled(y.data_ptr(), xd.data_ptr(), qt.data_ptr(), sd.data_ptr(), None,
                                           rd.data_ptr(), M, N, K, _lib.PS_BF16, wsp, ctypes.c_size_t(wsb),
                                           _lib.stream_ptr(dev))
            assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        outs.append(y)
    _lib.raise_on_device_error()
    assert torch.equal(outs[0], outs[1])
    ref = ops.quantized_linear(ops.round_bf16(x), q, scale, None) + ops.round_bf16(r)
    assert rel_err(outs[0].float().cpu().numpy(), ref) < REL_TOL


@pytest.mark.parametrize("M", [1, 7, 64, 576])
@pytest.mark.parametrize("IK", [(11008, 2048), (160, 256), (1376, 2048), (896, 640), (4744, 880), (160, 8192)])
def test_linear_swiglu_matches_oracle(dev, M, IK):
    """engine/model.py:188-190: silu(gate) * up from one linear over the
    row-interleaved gate|up int8 weight; also equal to the unfused gate|up
    linear followed by ps_silu_mul (same roundings) within the bf16 tolerance."""
    from pageserve_b200 import _lib
    from pageserve_b200.model import _interleave_rows
    from pageserve_b200.quantization import QuantizedWeight, linear_swiglu, w8a16_linear
    I, K = IK
    rng = np.random.default_rng(M * 7 + I)
    qg = rng.integers(-127, 128, size=(I, K)).astype(np.int8)
    qu = rng.integers(-127, 128, size=(I, K)).astype(np.int8)
    sg = rng.uniform(1e-3, 1e-2, size=(I, 1)).astype(np.float32)
    su = rng.uniform(1e-3, 1e-2, size=(I, 1)).astype(np.float32)
    x = rng.standard_normal((M, K), dtype=np.float32) * 0.5
    xb = _bf16(x, dev)
    wg = QuantizedWeight.from_quantized(torch.from_numpy(qg).to(dev), torch.from_numpy(sg).to(dev), torch.bfloat16)
    wu = QuantizedWeight.from_quantized(torch.from_numpy(qu).to(dev), torch.from_numpy(su).to(dev), torch.bfloat16)
    w_il = _interleave_rows(wg, wu, torch.bfloat16)
    y = linear_swiglu(xb, w_il)
    g = ops.round_bf16(ops.quantized_linear(ops.round_bf16(x), qg, sg))
    u = ops.round_bf16(ops.quantized_linear(ops.round_bf16(x), qu, su))
    ref = ops.silu(g) * u
    assert y.shape == (M, I)
    assert rel_err(y.float().cpu().numpy(), ref) < REL_TOL
    # unfused device path: gate|up linear, then ps_silu_mul
    gu = w8a16_linear(xb, torch.cat([wg.q, wu.q]), torch.cat([wg.scale, wu.scale]))
    act = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.load().ps_silu_mul(act.data_ptr(), gu.data_ptr(), M, I, _lib.PS_BF16, _lib.stream_ptr(dev)),
               "silu_mul")
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), act.float().cpu().numpy()) < 1e-2


def test_linear_swiglu_bf16_weight(dev):
    from pageserve_b200.model import _interleave_rows
    from pageserve_b200.quantization import linear_swiglu
    I, K, M = 384, 512, 40
    rng = np.random.default_rng(3)
    wg = rng.standard_normal((I, K), dtype=np.float32) * 0.05
    wu = rng.standard_normal((I, K), dtype=np.float32) * 0.05
    x = rng.standard_normal((M, K), dtype=np.float32)
    y = linear_swiglu(_bf16(x, dev), _interleave_rows(_bf16(wg, dev), _bf16(wu, dev), torch.bfloat16))
    g = ops.round_bf16(ops.linear(ops.round_bf16(x), ops.round_bf16(wg)))
    u = ops.round_bf16(ops.linear(ops.round_bf16(x), ops.round_bf16(wu)))
    assert rel_err(y.float().cpu().numpy(), ops.silu(g) * u) < REL_TOL
