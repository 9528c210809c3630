"""Generate the golden fixtures by running the UNMODIFIED reference.

Run once in a container that has the reference checkout (default path taken
from $PAGESERVE_REF):

    PAGESERVE_REF=<reference checkout> python tests/golden/make_golden.py

It imports the reference's own ``engine`` package (pure Python/torch, CPU,
float32), feeds it seeded inputs, and writes small ``.npz`` fixtures next to
this file. The fixtures hold the inputs and the reference's outputs, so the
tests that read them (tests/test_oracle_golden.py, tests/test_gpu_*.py) never
need the reference at run time.

Fixtures:
  ops_paged_attention.npz  write_kv / paged attention scenarios
                           (engine/paged_attention.py; the scenarios of the
                           reference's tests/test_paged_attention.py:40-140
                           plus larger GQA / chunked-prefill cases)
  ops_quant.npz            quantize_per_channel / dequantized linear
                           (engine/quantization.py)
  ops_norm_rope.npz        rms_norm, build_rope_cache, apply_rope
                           (engine/model.py:29-54)
  ops_tp.npz               column -> row parallel linear over 2 gloo ranks
                           (engine/tensor_parallel.py)
  model_tiny.npz           PagedCausalLM.forward_step on a tiny Qwen2 shape,
                           chunked prefill + decode over 3 sequences
  model_cfg1.npz           BASELINE config 1: the Qwen2.5-0.5B shape, int8,
                           fp32, 4 sequences at context 37/128/255/511
                           (summaries only: the logits are 4 x 151936)
  greedy_<name>.npz        greedy decode, 4 sequences x (prefill + 32 decode
                           steps), float32 and the reference's own bf16 picks
                           (cases.GREEDY_CASES)
  sched_trace.npz          the reference's scheduler + runner over a small
                           pool (chunked prefill, preemption) with a fake
                           model: per step the snapshot, entries and calls
"""

from __future__ import annotations

import os
import random
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from pageserve_b200 import synthetic  # noqa: E402

sys.path.insert(0, str(HERE))
import cases  # noqa: E402

REF = os.environ.get("PAGESERVE_REF")
if not REF:
    raise SystemExit("set PAGESERVE_REF to the reference checkout")
sys.path.insert(0, REF)

from engine import paged_attention as ref_pa  # noqa: E402
from engine import quantization as ref_q  # noqa: E402
from engine import model as ref_model  # noqa: E402

torch.set_num_threads(os.cpu_count() or 1)


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


# ------------------------------------------------------------ attention ----

def make_attention():
    """Run the reference's write_kv + paged_causal_attention_incremental over
    each case's chunks [(start_pos, T), ...] on one scrambled sequence."""
    res = {}
    for name in cases.ATTENTION_CASES:
        c = cases.attention_case(name)
        kc = torch.zeros(c["NB"], c["bs"], c["Hkv"], c["D"])
        vc = torch.zeros(c["NB"], c["bs"], c["Hkv"], c["D"])
        outs = []
        for (s, t) in c["chunks"]:
            ref_pa.write_kv(kc, vc, c["table"], c["bs"], s, _t(c["k"][s:s + t]), _t(c["v"][s:s + t]))
            o = ref_pa.paged_causal_attention_incremental(_t(c["q"][s:s + t]), kc, vc, c["table"], c["bs"], s)
            outs.append(o.numpy())
        out = np.concatenate(outs, axis=0)
        if cases.stores_full_output(name):
            res[f"{name}/out"] = out
        else:
            res[f"{name}/out_tail"] = out[-cases.TAIL_ROWS:]
            res[f"{name}/out_sum"] = out.astype(np.float64).sum(axis=(1, 2))
        if cases.stores_cache(name):
            res[f"{name}/k_cache"] = kc.numpy()
            res[f"{name}/v_cache"] = vc.numpy()
    np.savez_compressed(HERE / "ops_paged_attention.npz", **res)


# --------------------------------------------------------- quantization ----

def make_quant():
    rng = np.random.default_rng(99)
    w = rng.standard_normal((48, 96), dtype=np.float32)
    w[3] = 0.0                      # all-zero row: absmax clamp at 1e-8
    w[5] = np.linspace(-1, 1, 96, dtype=np.float32)
    w[7, :] = 0.5                   # every |w| at the absmax
    w[9] *= 1e-6                    # tiny row
    q, scale = ref_q.quantize_per_channel(_t(w))
    x = rng.standard_normal((8, 96), dtype=np.float32)
    b = rng.standard_normal((48,), dtype=np.float32)
    qw = ref_q.QuantizedWeight(_t(w))
    y = torch.nn.functional.linear(_t(x), qw.get(), _t(b))
    np.savez_compressed(HERE / "ops_quant.npz", w=w, q=q.numpy(), scale=scale.numpy(),
                        x=x, b=b, y=y.numpy(), storage_bytes=np.asarray(qw.storage_bytes))


# ------------------------------------------------------------ norm/rope ----

def make_norm_rope():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((6, 96), dtype=np.float32) * 3
    w = rng.standard_normal((96,), dtype=np.float32)
    y = ref_model.rms_norm(_t(x), _t(w), 1e-6)
    cos, sin = ref_model.build_rope_cache(64, 16, 1.0e4, "cpu", torch.float32)
    cos2, sin2 = ref_model.build_rope_cache(4096, 128, 1.0e6, "cpu", torch.float32)
    q = rng.standard_normal((5, 3, 16), dtype=np.float32)
    sp = 11
    qr = ref_model.apply_rope(_t(q), cos[sp:sp + 5], sin[sp:sp + 5])
    np.savez_compressed(HERE / "ops_norm_rope.npz", x=x, w=w, y=y.numpy(), cos=cos.numpy(), sin=sin.numpy(),
                        cos_4096_128=cos2.numpy()[::97], sin_4096_128=sin2.numpy()[::97],
                        q=q, start_pos=np.asarray(sp), q_rope=qr.numpy())


# ------------------------------------------------------------------- TP ----

def _tp_worker(rank, world_size, sync_file, data_file, result_file):
    import torch.distributed as dist
    from engine.tensor_parallel import column_parallel_linear, row_parallel_linear
    dist.init_process_group("gloo", rank=rank, world_size=world_size, init_method=f"file://{sync_file}")
    d = torch.load(data_file, weights_only=True)
    h = column_parallel_linear(d["x"], d["w1"], rank, world_size)
    out = row_parallel_linear(h, d["w2"], rank, world_size)
    torch.save({"h": h, "out": out}, f"{result_file}.{rank}")
    dist.destroy_process_group()


def make_tp():
    import torch.multiprocessing as mp
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 16), dtype=np.float32)
    w1 = rng.standard_normal((8, 16), dtype=np.float32)
    w2 = rng.standard_normal((16, 8), dtype=np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        data = os.path.join(tmp, "d.pt")
        torch.save({"x": _t(x), "w1": _t(w1), "w2": _t(w2)}, data)
        mp.spawn(_tp_worker, args=(2, os.path.join(tmp, "sync"), data, os.path.join(tmp, "r")), nprocs=2, join=True)
        r0 = torch.load(os.path.join(tmp, "r.0"), weights_only=True)
        r1 = torch.load(os.path.join(tmp, "r.1"), weights_only=True)
    np.savez_compressed(HERE / "ops_tp.npz", x=x, w1=w1, w2=w2, h0=r0["h"].numpy(), h1=r1["h"].numpy(),
                        out0=r0["out"].numpy(), out1=r1["out"].numpy())


# ---------------------------------------------------------------- model ----

def _save_checkpoint(shape, sd_np, directory):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(
        vocab_size=shape.vocab, hidden_size=shape.hidden, intermediate_size=shape.intermediate,
        num_hidden_layers=shape.num_layers, num_attention_heads=shape.num_heads,
        num_key_value_heads=shape.num_kv_heads, max_position_embeddings=shape.max_position,
        rope_theta=shape.rope_theta, rms_norm_eps=shape.rms_eps, tie_word_embeddings=shape.tie_embeddings)
    m = Qwen2ForCausalLM(cfg)
    sd = {k: _t(v) for k, v in sd_np.items()}
    if shape.tie_embeddings:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = m.load_state_dict(sd, strict=False)
    assert not unexpected and all(k == "lm_head.weight" for k in missing), (missing, unexpected)
    m.save_pretrained(directory)


def make_tiny_model():
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=5, perturb_norms_biases=True)
    rng = np.random.default_rng(21)
    NB, bs = 40, 4
    ids = list(range(NB))
    random.Random(4).shuffle(ids)
    # three sequences with disjoint scrambled block tables
    prompts = [rng.integers(0, shape.vocab, size=n).astype(np.int64) for n in (13, 6, 22)]
    tables = [ids[0:10], ids[10:20], ids[20:40]]
    out = {"seed": np.asarray(5)}
    with tempfile.TemporaryDirectory() as tmp:
        _save_checkpoint(shape, sd, tmp)
        for quant in (True, False):
            m = ref_model.PagedCausalLM(tmp, device="cpu", dtype=torch.float32, quantize=quant)
            m.allocate_kv_cache(NB, bs)
            steps = []   # (seq, start_pos, token ids)
            logits = []
            # chunked prefill with chunk 5 interleaved across sequences, then decodes
            pos = [0, 0, 0]
            chunk = 5
            active = True
            while active:
                active = False
                for s in range(3):
                    if pos[s] < len(prompts[s]):
                        t = prompts[s][pos[s]:pos[s] + chunk]
                        steps.append((s, pos[s], t))
                        pos[s] += len(t)
                        active = True
            nxt = {}
            for s, sp, t in steps:
                lg = m.forward_step(_t(t), tables[s], sp)
                logits.append(lg.numpy())
                if sp + len(t) == len(prompts[s]):
                    nxt[s] = int(lg[-1].argmax())
            # 4 greedy decode steps per sequence
            for _ in range(4):
                for s in range(3):
                    sp = pos[s]
                    t = np.asarray([nxt[s]], np.int64)
                    steps.append((s, sp, t))
                    lg = m.forward_step(_t(t), tables[s], sp)
                    logits.append(lg.numpy())
                    nxt[s] = int(lg[-1].argmax())
                    pos[s] += 1
            tag = "q" if quant else "f"
            out[f"{tag}/step_seq"] = np.asarray([s for s, _, _ in steps], np.int32)
            out[f"{tag}/step_pos"] = np.asarray([p for _, p, _ in steps], np.int32)
            out[f"{tag}/step_len"] = np.asarray([len(t) for _, _, t in steps], np.int32)
            out[f"{tag}/step_tokens"] = np.concatenate([t for _, _, t in steps]).astype(np.int64)
            out[f"{tag}/logits"] = np.concatenate(logits, axis=0)
            out[f"{tag}/k_cache"] = m.k_cache.numpy()
            out[f"{tag}/v_cache"] = m.v_cache.numpy()
    out["tables"] = np.asarray([t + [-1] * (20 - len(t)) for t in tables], np.int32)
    out["dims"] = np.asarray([NB, bs], np.int32)
    np.savez_compressed(HERE / "model_tiny.npz", **out)


def make_cfg1():
    shape = synthetic.QWEN25_0_5B
    sd = synthetic.generate_state_dict(shape, seed=0)
    prompts, tables = cases.cfg1_inputs(shape.vocab)
    with tempfile.TemporaryDirectory() as tmp:
        _save_checkpoint(shape, sd, tmp)
        del sd
        m = ref_model.PagedCausalLM(tmp, device="cpu", dtype=torch.float32, quantize=True)
    m.allocate_kv_cache(256, 16)
    res = {}
    for i, (p, tab) in enumerate(zip(prompts, tables)):
        ctx = len(p)
        with torch.no_grad():
            lp = m.forward_step(_t(p[:-1]), tab, 0)            # prefill ctx-1 tokens
            ld = m.forward_step(_t(p[-1:]), tab, ctx - 1)       # one decode token
        for tag, lg in (("prefill", lp[-1]), ("decode", ld[-1])):
            lg = lg.numpy().astype(np.float32)
            order = np.argsort(-lg)[:16]
            res[f"{i}/{tag}/argmax"] = np.asarray(int(lg.argmax()))
            res[f"{i}/{tag}/top_idx"] = order.astype(np.int64)
            res[f"{i}/{tag}/top_val"] = lg[order]
            res[f"{i}/{tag}/sample"] = lg[::cases.CFG1_STRIDE]
            res[f"{i}/{tag}/sum"] = np.asarray(lg.astype(np.float64).sum())
        # written KV rows of this sequence, summarised per layer
        slots = [(tab[pp // 16], pp % 16) for pp in range(ctx)]
        kk = torch.stack([m.k_cache[:, b, o] for b, o in slots], dim=1).numpy()  # (L, ctx, Hkv, D)
        vv = torch.stack([m.v_cache[:, b, o] for b, o in slots], dim=1).numpy()
        res[f"{i}/k_layer_sum"] = kk.astype(np.float64).sum(axis=(1, 2, 3))
        res[f"{i}/v_layer_sum"] = vv.astype(np.float64).sum(axis=(1, 2, 3))
        res[f"{i}/k_layer_abs"] = np.abs(kk).astype(np.float64).sum(axis=(1, 2, 3))
        res[f"{i}/k_last_layer_rows"] = kk[-1, ::7]
        res[f"{i}/v_last_layer_rows"] = vv[-1, ::7]
    # the reference's own bf16 path (its GPU dtype) on the same inputs: its picks
    with tempfile.TemporaryDirectory() as tmp:
        sd = synthetic.generate_state_dict(shape, seed=0)
        _save_checkpoint(shape, sd, tmp)
        del sd
        mb = ref_model.PagedCausalLM(tmp, device="cpu", dtype=torch.bfloat16, quantize=True)
    mb.allocate_kv_cache(256, 16)
    for i, (p, tab) in enumerate(zip(prompts, tables)):
        ctx = len(p)
        with torch.no_grad():
            lp = mb.forward_step(_t(p[:-1]), tab, 0)
            ld = mb.forward_step(_t(p[-1:]), tab, ctx - 1)
        res[f"{i}/prefill/argmax_bf16"] = np.asarray(int(lp[-1].argmax()))
        res[f"{i}/decode/argmax_bf16"] = np.asarray(int(ld[-1].argmax()))
    for i, (p, tab) in enumerate(zip(prompts, tables)):
        res[f"{i}/tokens"] = p
        res[f"{i}/table"] = np.asarray(tab, np.int32)
    res["ctx"] = np.asarray(cases.CFG1_CTX, np.int32)
    res["stride"] = np.asarray(cases.CFG1_STRIDE)
    np.savez_compressed(HERE / "model_cfg1.npz", **res)


def make_greedy():
    """Greedy decode by the reference (engine/model.py:149-193 driven one
    sequence at a time, as engine/runner.py:65-79 and
    scripts/verify_end_to_end.py:63-91 do): each sequence prefills its prompt,
    then takes cases.GREEDY_STEPS decode steps feeding back
    ``int(logits[-1].argmax())``. Per decision the fixture keeps the chosen
    token, the reference's top-16 (ids, logits) and a strided sample of the
    logits, so a test can tell a near-tie flip from a real one. A second run of
    the reference in bfloat16 (its GPU dtype), fed the float32 run's tokens,
    records its own pick at every decision (``gen_bf16``)."""
    for name, (shape, seed, perturb, ctxs) in cases.GREEDY_CASES.items():
        sd = synthetic.generate_state_dict(shape, seed=seed, perturb_norms_biases=perturb)
        prompts, tables = cases.greedy_inputs(name)
        with tempfile.TemporaryDirectory() as tmp:
            _save_checkpoint(shape, sd, tmp)
            del sd
            m = ref_model.PagedCausalLM(tmp, device="cpu", dtype=torch.float32, quantize=True)
        m.allocate_kv_cache(cases.GREEDY_POOL, 16)
        S = cases.GREEDY_STEPS + 1
        gen = np.zeros((len(prompts), S), np.int64)
        top_idx = np.zeros((len(prompts), S, 16), np.int64)
        top_val = np.zeros((len(prompts), S, 16), np.float32)
        samples = []
        for i, (p, tab) in enumerate(zip(prompts, tables)):
            rows = []
            with torch.no_grad():
                lg = m.forward_step(_t(p), tab, 0)[-1]
                for t in range(S):
                    lgn = lg.numpy().astype(np.float32)
                    order = np.argsort(-lgn, kind="stable")[:16]
                    tok = int(lg.argmax())
                    gen[i, t] = tok
                    top_idx[i, t] = order
                    top_val[i, t] = lgn[order]
                    rows.append(lgn[::cases.GREEDY_STRIDE])
                    if t + 1 < S:
                        lg = m.forward_step(torch.tensor([tok]), tab, len(p) + t)[-1]
            samples.append(np.stack(rows))
            print(f"  {name} seq {i}: ctx {len(p)} -> {gen[i].tolist()}", flush=True)
        # The reference's own bf16 path on the same decisions (teacher forced
        # with the float32 run's tokens): its greedy pick at every decision.
        with tempfile.TemporaryDirectory() as tmp:
            sd = synthetic.generate_state_dict(shape, seed=seed, perturb_norms_biases=perturb)
            _save_checkpoint(shape, sd, tmp)
            del sd
            mb = ref_model.PagedCausalLM(tmp, device="cpu", dtype=torch.bfloat16, quantize=True)
        mb.allocate_kv_cache(cases.GREEDY_POOL, 16)
        gen_bf16 = np.zeros_like(gen)
        for i, (p, tab) in enumerate(zip(prompts, tables)):
            with torch.no_grad():
                lg = mb.forward_step(_t(p), tab, 0)[-1]
                for t in range(S):
                    gen_bf16[i, t] = int(lg.argmax())
                    if t + 1 < S:
                        lg = mb.forward_step(torch.tensor([int(gen[i, t])]), tab, len(p) + t)[-1]
            print(f"  {name} seq {i} bf16: {int((gen_bf16[i] != gen[i]).sum())} of {S} decisions differ", flush=True)
        res = {"gen": gen, "top_idx": top_idx, "top_val": top_val, "sample": np.stack(samples),
               "stride": np.asarray(cases.GREEDY_STRIDE), "gen_bf16": gen_bf16}
        for i, (p, tab) in enumerate(zip(prompts, tables)):
            res[f"{i}/tokens"] = p
            res[f"{i}/table"] = np.asarray(tab, np.int32)
        np.savez_compressed(HERE / f"greedy_{name}.npz", **res)


def make_sched_trace():
    """The reference's own continuous batching (engine/scheduler.py +
    engine/runner.py's ContinuousBatchingRunner, unmodified) over a small
    block pool that forces chunked prefill, preemption and recompute, with a
    deterministic fake model (cases.fake_next_token). Records, per scheduler
    step, the running sequences' state the runner snapshots before step(), the
    batch entries, and every process_chunk call with the token it returned."""
    import threading

    from engine.block_allocator import BlockAllocator
    from engine.runner import ContinuousBatchingRunner
    from engine.scheduler import Scheduler
    from engine.sequence import Sequence

    steps = []
    calls = []
    lock = threading.Lock()

    class RecordingScheduler(Scheduler):
        def step(self):
            snap = [(s.seq_id, s.num_prompt_tokens_processed, len(s.output_tokens)) for s in self.running]
            batch = super().step()
            steps.append({"snapshot": snap, "entries": [(e.seq.seq_id, e.chunk, e.produces_token) for e in batch]})
            return batch

    def process_chunk(input_ids, block_table, start_pos):
        tok = cases.fake_next_token(input_ids, start_pos)
        with lock:
            calls.append((list(input_ids), list(block_table), int(start_pos), tok, len(steps) - 1))
        return tok

    spec = cases.SCHED_TRACE
    alloc = BlockAllocator(num_blocks=spec["num_blocks"], block_size=spec["block_size"])
    sched = RecordingScheduler(alloc, block_size=spec["block_size"], max_batch_size=spec["max_batch_size"],
                               token_budget=spec["token_budget"])
    prompts = cases.sched_trace_prompts()
    seqs = [Sequence(prompt_tokens=list(p), max_new_tokens=n) for p, n in zip(prompts, spec["max_new"])]
    id_of = {s.seq_id: i for i, s in enumerate(seqs)}  # global seq ids -> request index
    for s in seqs:  # every request present before the runner's thread starts: a deterministic trace
        sched.add_request(s)
    runner = ContinuousBatchingRunner(sched, process_chunk)
    for s in seqs:
        runner.wait_until_finished(s, timeout=60)
    runner.stop()
    out = {"n_steps": np.asarray(len(steps))}
    for k, st in enumerate(steps):
        out[f"{k}/snapshot"] = np.asarray([(id_of[a], b, c) for a, b, c in st["snapshot"]], np.int64).reshape(-1, 3)
        out[f"{k}/entries"] = np.asarray([(id_of[a], b, int(c)) for a, b, c in st["entries"]], np.int64).reshape(-1, 3)
    for j, (ids, table, start, tok, k) in enumerate(calls):
        out[f"call{j}/ids"] = np.asarray(ids, np.int64)
        out[f"call{j}/table"] = np.asarray(table, np.int64)
        out[f"call{j}/meta"] = np.asarray([start, tok, k], np.int64)
    out["n_calls"] = np.asarray(len(calls))
    for i, s in enumerate(seqs):
        out[f"out{i}"] = np.asarray(s.output_tokens, np.int64)
    np.savez_compressed(HERE / "sched_trace.npz", **out)
    print(f"  {len(steps)} scheduler steps, {len(calls)} process_chunk calls", flush=True)


if __name__ == "__main__":
    which = sys.argv[1:] or ["attention", "quant", "norm_rope", "tp", "tiny", "cfg1", "greedy", "sched"]
    for w in which:
        print("generating", w, flush=True)
        {"attention": make_attention, "quant": make_quant, "norm_rope": make_norm_rope, "tp": make_tp,
         "tiny": make_tiny_model, "cfg1": make_cfg1, "greedy": make_greedy, "sched": make_sched_trace}[w]()
    print("done")
