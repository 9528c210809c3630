"""Pins the numpy oracle to the reference: every fixture under tests/golden/
was produced by the unmodified reference (tests/golden/make_golden.py); the
oracle must reproduce it on the same inputs (CPU, float32)."""

import numpy as np
import pytest

import cases
from oracle import ops
from oracle.model import OracleCausalLM
from pageserve_b200 import synthetic

from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(GOLDEN / name, allow_pickle=False)


@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_oracle_paged_attention_matches_reference(name):
    g = _load("ops_paged_attention.npz")
    c = cases.attention_case(name)
    kc = np.zeros((c["NB"], c["bs"], c["Hkv"], c["D"]), np.float32)
    vc = np.zeros_like(kc)
    outs = []
    for s, t in c["chunks"]:
        ops.write_kv(kc, vc, c["table"], c["bs"], s, c["k"][s:s + t], c["v"][s:s + t])
        outs.append(ops.paged_causal_attention_incremental(c["q"][s:s + t], kc, vc, c["table"], c["bs"], s))
    out = np.concatenate(outs, axis=0)
    if cases.stores_cache(name):
        # write_kv is a copy: bit-exact against the reference's cache.
        assert np.array_equal(kc, g[f"{name}/k_cache"])
        assert np.array_equal(vc, g[f"{name}/v_cache"])
    if cases.stores_full_output(name):
        np.testing.assert_allclose(out, g[f"{name}/out"], atol=1e-5, rtol=0)
    else:
        np.testing.assert_allclose(out[-cases.TAIL_ROWS:], g[f"{name}/out_tail"], atol=1e-5, rtol=0)
        np.testing.assert_allclose(out.astype(np.float64).sum(axis=(1, 2)), g[f"{name}/out_sum"], atol=1e-3, rtol=0)


def test_oracle_gather_raises_index_error_on_short_table():
    kc = np.zeros((4, 4, 1, 2), np.float32)
    with pytest.raises(IndexError):
        ops.gather_kv(kc, kc, [0], 4, 5)
    with pytest.raises(IndexError):
        ops.write_kv(kc, kc, [0], 4, 4, np.zeros((1, 1, 2), np.float32), np.zeros((1, 1, 2), np.float32))


def test_oracle_quantization_bit_exact():
    g = _load("ops_quant.npz")
    q, scale = ops.quantize_per_channel(g["w"])
    assert q.dtype == np.int8 and scale.shape == (48, 1)
    assert np.array_equal(q, g["q"])
    assert np.array_equal(scale, g["scale"])
    y = ops.quantized_linear(g["x"], q, scale, g["b"])
    np.testing.assert_allclose(y, g["y"], atol=1e-5, rtol=0)
    assert q.nbytes + scale.nbytes == int(g["storage_bytes"])


def test_oracle_norm_rope():
    g = _load("ops_norm_rope.npz")
    np.testing.assert_allclose(ops.rms_norm(g["x"], g["w"], 1e-6), g["y"], atol=1e-5, rtol=1e-6)
    cos, sin = ops.build_rope_cache(64, 16, 1.0e4)
    np.testing.assert_allclose(cos, g["cos"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(sin, g["sin"], atol=2e-6, rtol=0)
    cos2, sin2 = ops.build_rope_cache(4096, 128, 1.0e6)
    # large angles: float32 argument rounding dominates; both sides use the
    # same float32 angle, so the values agree to a few ulps of the angle.
    np.testing.assert_allclose(cos2[::97], g["cos_4096_128"], atol=2e-3, rtol=0)
    np.testing.assert_allclose(sin2[::97], g["sin_4096_128"], atol=2e-3, rtol=0)
    sp = int(g["start_pos"])
    qr = ops.apply_rope(g["q"], cos[sp:sp + 5], sin[sp:sp + 5])
    np.testing.assert_allclose(qr, g["q_rope"], atol=1e-5, rtol=0)


def test_oracle_tensor_parallel():
    g = _load("ops_tp.npz")
    h = [ops.column_parallel_linear(g["x"], g["w1"], r, 2) for r in range(2)]
    np.testing.assert_allclose(h[0], g["h0"], atol=1e-5)
    np.testing.assert_allclose(h[1], g["h1"], atol=1e-5)
    out = ops.row_parallel_linear_all_ranks(h, g["w2"])
    np.testing.assert_allclose(out, g["out0"], atol=1e-4)
    np.testing.assert_allclose(out, g["out1"], atol=1e-4)
    with pytest.raises(AssertionError):
        ops.column_parallel_linear(g["x"], g["w1"][:7], 0, 2)


def _run_tiny(quant):
    g = _load("model_tiny.npz")
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=int(g["seed"]), perturb_norms_biases=True)
    m = OracleCausalLM(sd, shape, quantize=quant)
    NB, bs = (int(x) for x in g["dims"])
    m.allocate_kv_cache(NB, bs)
    tag = "q" if quant else "f"
    tables = [[int(b) for b in row if b >= 0] for row in g["tables"]]
    toks = g[f"{tag}/step_tokens"]
    at = 0
    logits = []
    for s, p, n in zip(g[f"{tag}/step_seq"], g[f"{tag}/step_pos"], g[f"{tag}/step_len"]):
        logits.append(m.forward_step(toks[at:at + n], tables[s], int(p)))
        at += n
    return g, tag, m, np.concatenate(logits, axis=0)


@pytest.mark.parametrize("quant", [True, False])
def test_oracle_tiny_model_matches_reference(quant):
    g, tag, m, logits = _run_tiny(quant)
    np.testing.assert_allclose(logits, g[f"{tag}/logits"], atol=2e-4, rtol=0)
    assert np.array_equal(logits.argmax(-1), g[f"{tag}/logits"].argmax(-1))
    np.testing.assert_allclose(m.k_cache, g[f"{tag}/k_cache"], atol=2e-5, rtol=0)
    np.testing.assert_allclose(m.v_cache, g[f"{tag}/v_cache"], atol=2e-5, rtol=0)


@pytest.mark.slow
def test_oracle_config1_matches_reference():
    """BASELINE config 1 (Qwen2.5-0.5B shape, int8, fp32), 4 sequences."""
    path = GOLDEN / "model_cfg1.npz"
    if not path.exists():
        pytest.skip("model_cfg1.npz not generated")
    g = np.load(path)
    shape = synthetic.QWEN25_0_5B
    sd = synthetic.generate_state_dict(shape, seed=0)
    m = OracleCausalLM(sd, shape, quantize=True, max_position=1024)
    del sd
    m.allocate_kv_cache(256, 16)
    stride = int(g["stride"])
    for i in range(len(g["ctx"])):
        p = g[f"{i}/tokens"]
        tab = [int(b) for b in g[f"{i}/table"]]
        ctx = len(p)
        lp = m.forward_step(p[:-1], tab, 0, logits_rows=[ctx - 2])[-1]
        ld = m.forward_step(p[-1:], tab, ctx - 1)[-1]
        for tag, lg in (("prefill", lp), ("decode", ld)):
            assert int(lg.argmax()) == int(g[f"{i}/{tag}/argmax"])
            np.testing.assert_allclose(lg[::stride], g[f"{i}/{tag}/sample"], atol=2e-4, rtol=0)
            np.testing.assert_allclose(lg[g[f"{i}/{tag}/top_idx"]], g[f"{i}/{tag}/top_val"], atol=2e-4, rtol=0)
        kk = np.stack([m.k_cache[:, tab[pp // 16], pp % 16] for pp in range(ctx)], axis=1)
        np.testing.assert_allclose(kk.astype(np.float64).sum(axis=(1, 2, 3)), g[f"{i}/k_layer_sum"], atol=5e-2, rtol=1e-5)
        np.testing.assert_allclose(kk[-1, ::7], g[f"{i}/k_last_layer_rows"], atol=5e-4, rtol=0)


@pytest.mark.slow
@pytest.mark.parametrize("name,seq,steps", [("cfg1", 0, 12), ("3b4", 0, 6)])
def test_oracle_greedy_decode_matches_reference(name, seq, steps):
    """The reference's greedy decode (tests/golden/greedy_*.npz), teacher
    forced on the oracle: the same pick at every decision and the same top-16
    logits (float32 against float32: only summation order differs)."""
    g = np.load(GOLDEN / f"greedy_{name}.npz")
    shape, seed, perturb, _ = cases.GREEDY_CASES[name]
    prompts, tables = cases.greedy_inputs(name)
    sd = synthetic.generate_state_dict(shape, seed=seed, perturb_norms_biases=perturb)
    m = OracleCausalLM(sd, shape, quantize=True, max_position=2048)
    del sd
    m.allocate_kv_cache(cases.GREEDY_POOL, 16)
    p, tab = prompts[seq], tables[seq]
    lg = m.forward_step(p, tab, 0, logits_rows=[len(p) - 1])[-1]
    for t in range(steps):
        assert int(lg.argmax()) == int(g["gen"][seq, t]), f"decision {t}"
        np.testing.assert_allclose(lg[g["top_idx"][seq, t]], g["top_val"][seq, t], atol=2e-4, rtol=0)
        np.testing.assert_allclose(lg[::int(g["stride"])], g["sample"][seq, t], atol=2e-4, rtol=0)
        lg = m.forward_step([int(g["gen"][seq, t])], tab, len(p) + t)[-1]
