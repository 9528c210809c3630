"""Benchmark: decode tok/s of a Qwen2.5-3B-shape W8A16 model, batch 64.

Workload (the configuration the headline metric is quoted
on): one mixed scheduler step of a random-init Qwen2.5-3B-shaped decoder
(36 layers, hidden 2048, 16/2 heads, head_dim 128, intermediate 11008, vocab
151936, tied bf16 lm_head, int8 per-channel layer weights, bf16 KV, block
size 16): 64 decode sequences at context 2048 plus one 512-token prefill
chunk. A "step" is one pass of the whole hot path over that batch; the
decode throughput is 64 tokens per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl pageserve_b200|reference]

value: decode tok/s over K CUDA-graph replays of the step, inputs resident in
HBM (the step streams ~8 GB of weights + KV, far larger than the 126 MB L2,
so no flush is needed between steps).
e2e: the same metric through the public step API (StepGraph.run): per step a
host->device copy of token ids + metadata from pinned memory and a
device->host read of the 65 greedy next tokens.
--gpus N > 1: Megatron tensor parallelism over N ranks (one process per GPU,
NCCL all-reduce after o_proj and down_proj, vocab-parallel lm_head): one
model serving the same 64 sequences, so the work is fixed (strong scaling).
--replicas: N independent single-GPU replicas instead (weak scaling).
--impl reference: the reference algorithm's CPU path (the oracle port of
engine/model.py, one forward_step per sequence as engine/runner.py:65-79
does), on a bounded sample of the same workload, all host threads.
--config 5: BASELINE config 5 instead (Qwen2.5-32B shape, 64 layers, hidden
5120, 40/8 heads, intermediate 27648, untied vocab 152064, int8): a decode
step of 128 sequences at context 4096, tensor parallel over --gpus N ranks
(one GPU holds the whole model and its 137 GB KV cache at N = 1).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (Qwen2.5-3B-shape W8A16, bs64)"
UNIT = "tok/s"
N_DECODE, CTX, PREFILL = 64, 2048, 512
BLOCK = 16
CONFIG = 4
SHAPE_NAME = "qwen2.5-3b"


def _use_config5():
    """32B-shape int8 decode, B = 128 at context 4096."""
    global METRIC, N_DECODE, CTX, PREFILL, CONFIG, SHAPE_NAME
    METRIC = "decode tok/s (Qwen2.5-32B-shape W8A16 TP, bs128 @ctx 4096)"
    N_DECODE, CTX, PREFILL, CONFIG, SHAPE_NAME = 128, 4096, 0, 5, "qwen2.5-32b"


TP_COMM_NAMES = {
    "fused": "fused one-shot peer-memory push (o_proj/down -> next RMSNorm)",
    "fused2": "fused two-shot: GEMM scatters column slices to owners, owner reduces + all-gathers the residual, "
              "local RMSNorm",
    "nccl": "NCCL all_reduce",
}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _shape():
    from pageserve_b200 import synthetic
    return synthetic.SHAPES[SHAPE_NAME]


def _config(extra=None):
    if CONFIG == 5:
        wl = ("BASELINE config 5: Qwen2.5-32B-shape int8 decode step, 128 seqs @ctx 4096, block 16, "
              "tensor parallel over the job's GPUs")
    elif PREFILL:
        wl = ("BASELINE config 4: Qwen2.5-3B-shape int8 mixed step, 64 decode seqs @ctx 2048 "
              f"+ one {PREFILL}-token prefill chunk, block 16")
    else:
        wl = ("Qwen2.5-3B-shape int8 decode-only step (config 4 without its prefill chunk): 64 decode seqs "
              "@ctx 2048, block 16")
    c = {"workload": wl,
         "model": f"{SHAPE_NAME}-shape (random init)", "layers": _shape().num_layers, "global_batch": N_DECODE,
         "prefill_tokens_per_step": PREFILL, "seq_len": CTX, "kv_dtype": "bf16", "weights": "int8 per-channel",
         "l2": ("inputs larger than L2 (~8 GB of weights + KV streamed per step)" if CONFIG == 4 else
                "inputs larger than L2 (~170 GB of weights + KV per step over all ranks)")}
    if extra:
        c.update(extra)
    return c


# --------------------------------------------------------------- clocks ----

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        fd, name = tempfile.mkstemp(prefix=f"ps_clocks_{gpu_index}_", suffix=".csv")
        os.close(fd)
        self.path = Path(name)

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
            # start timing only once the sampler writes (nvidia-smi takes ~0.1-1 s to come up)
            t0 = time.time()
            while time.time() - t0 < 3.0 and self.path.stat().st_size == 0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.proc or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        try:
            self.path.unlink()
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- workload ----

def build_workload(device, seed=0, tp=None, tp_comm="auto"):
    import numpy as np
    import torch

    from pageserve_b200 import synthetic
    from pageserve_b200.model import PagedCausalLM

    shape = synthetic.SHAPES[SHAPE_NAME]
    sd = synthetic.TorchStateDict(shape, seed=seed, device=device)
    m = PagedCausalLM.from_state_dict(sd, shape, device=device, dtype=torch.bfloat16, quantize=True,
                                      max_position=max(4096, CTX), tp=tp, tp_comm=tp_comm, tp_max_tokens=N_DECODE + PREFILL)
    del sd
    torch.cuda.empty_cache()
    nblk_dec = CTX // BLOCK
    nblk_pre = PREFILL // BLOCK
    num_blocks = N_DECODE * nblk_dec + nblk_pre + 64
    m.allocate_kv_cache(num_blocks, BLOCK)
    g = torch.Generator(device=device)
    g.manual_seed(seed + 7)
    for c in (m.k_cache, m.v_cache):
        c.normal_(0.0, 1.0, generator=g)
    rng = np.random.default_rng(seed)
    perm = rng.permutation(num_blocks)
    tables, at = [], 0
    for _ in range(N_DECODE):
        tables.append(perm[at:at + nblk_dec].tolist())
        at += nblk_dec
    if PREFILL:
        tables.append(perm[at:at + nblk_pre].tolist())
    q_lens = [1] * N_DECODE + ([PREFILL] if PREFILL else [])
    start_pos = [CTX - 1] * N_DECODE + ([0] if PREFILL else [])
    ids = rng.integers(0, shape.vocab, size=N_DECODE + PREFILL).astype(np.int64)
    return m, dict(q_lens=q_lens, start_pos=start_pos, tables=tables, ids=ids, shape=shape)


def time_events(fn, iters):
    """Device time of one ``fn`` call (ms): ``iters`` calls captured once into
    a CUDA graph, the graph replayed between CUDA events on the current
    stream (the way the step runs them, without host launch gaps)."""
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    g.replay()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / iters
    del g
    return ms


# ncu summaries (profiles/) of the step's kernel classes: same kernel, same shape
PROFILE_OF = {"gate_up": "linear_tc_gate_up_swiglu_M576.md", "down": "linear_tc_down_M576.md",
              "qkv": "linear_tc_qkv_M576.md", "attn_decode": "decode_tma_cfg4.md",
              "attn_prefill": "prefill_tc_T512.md"}


def profile_traffic(kernel):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch of `kernel`
    from its committed ncu summary (None when there is none)."""
    name = PROFILE_OF.get(kernel)
    if not name or PREFILL != 512 or CONFIG != 4:  # the captures are of the config-4 shapes (576 tokens)
        return None, None
    path = ROOT / "profiles" / name
    try:
        for line in path.read_text().splitlines():
            cells = [c.strip() for c in line.strip().strip("|").split("|")]
            if len(cells) >= 2 and cells[0] == "traffic_bytes_per_launch":
                return int(cells[1]), f"profiles/{name} (ncu dram__bytes_read.sum + dram__bytes_write.sum)"
    except (OSError, ValueError):
        pass
    return None, None


def kernel_breakdown(m, w, peaks):
    """Each main kernel of the step timed alone (CUDA-graph replay between
    CUDA events), rotating over the layers' weights / caches so nothing
    is served from L2."""
    import torch

    from pageserve_b200.paged_attention import AttentionWorkspace, paged_attention
    from pageserve_b200.quantization import LinearWorkspace, linear16, linear_swiglu

    dev = m.device
    T = N_DECODE + PREFILL
    L = len(m.fused)
    H, I = m.hidden_size, m.intermediate_size
    x_h = torch.randn(T, H, device=dev, dtype=torch.bfloat16)
    x_i = torch.randn(T, I, device=dev, dtype=torch.bfloat16)
    x_a = torch.randn(T, m.heads_local * m.head_dim, device=dev, dtype=torch.bfloat16)
    ws = LinearWorkspace()
    res = {}

    def lin(name, x, get_w, swiglu=False):
        outs = {}
        ctr = [0]

        def f():
            wgt = get_w(m.fused[ctr[0] % L])
            ctr[0] += 1
            if swiglu:  # the gate|up linear with SiLU*up in its epilogue, as the step runs it
                outs["y"] = linear_swiglu(x, wgt)
            else:  # the step's path: the tiled int8 copy (the model keeps no row-major one)
                outs["y"] = wgt.linear(x, workspace=ws)
        f()
        ms = time_events(f, 2 * L)
        wgt = get_w(m.fused[0])
        N, K = wgt.shape
        M = x.shape[0]
        flops = 2.0 * M * N * K
        byts = N * K + 4 * N + 2 * M * K + 2 * M * (N // 2 if swiglu else N)
        res[name] = {"ms": ms, "M": M, "N": N, "K": K, "tflops": flops / ms / 1e9, "gbs": byts / ms / 1e6,
                     "flops": flops, "bytes": byts}

    lin("qkv", x_h, lambda f: f.qkv)
    lin("o_proj", x_a, lambda f: f.o)
    lin("gate_up", x_h, lambda f: f.gate_up, swiglu=True)
    lin("down", x_i, lambda f: f.down)
    # lm_head on the 65 sampled rows
    xl = torch.randn(N_DECODE + 1, H, device=dev, dtype=torch.bfloat16)
    f = lambda: linear16(xl, m.lm_head_w, workspace=ws)  # noqa: E731
    f()
    ms = time_events(f, 5)
    V = m.lm_head_w.shape[0]
    byts = V * H * 2 + 2 * xl.shape[0] * (H + V)
    res["lm_head"] = {"ms": ms, "M": xl.shape[0], "N": V, "K": H, "gbs": byts / ms / 1e6, "bytes": byts,
                      "tflops": 2.0 * xl.shape[0] * V * H / ms / 1e9, "flops": 2.0 * xl.shape[0] * V * H}
    # decode attention: the decode sequences at their context, rotating over layer caches
    meta = m.make_meta([1] * N_DECODE, [CTX - 1] * N_DECODE, w["tables"][:N_DECODE])
    q = torch.randn(N_DECODE, m.heads_local, m.head_dim, device=dev, dtype=torch.bfloat16)
    aws = AttentionWorkspace()
    ctr = [0]

    def att():
        li = ctr[0] % L
        ctr[0] += 1
        paged_attention(q, m.k_cache[li], m.v_cache[li], meta.block_tables, meta.cu_q, meta.start_pos, 1, CTX,
                        workspace=aws)
    att()
    ms = time_events(att, 2 * L)
    kv = N_DECODE * CTX * m.kv_heads_local * m.head_dim * 2 * 2
    byts = kv + 2 * 2 * N_DECODE * m.heads_local * m.head_dim + 4 * N_DECODE * (CTX // BLOCK)
    res["attn_decode"] = {"ms": ms, "gbs": byts / ms / 1e6, "bytes": byts}
    if not PREFILL:
        return res
    # the prefill chunk at position 0 (causal), rotating over layer caches
    pmeta = m.make_meta([PREFILL], [0], w["tables"][N_DECODE:])
    qp = torch.randn(PREFILL, m.heads_local, m.head_dim, device=dev, dtype=torch.bfloat16)
    ctr2 = [0]

    def attp():
        li = ctr2[0] % L
        ctr2[0] += 1
        paged_attention(qp, m.k_cache[li], m.v_cache[li], pmeta.block_tables, pmeta.cu_q, pmeta.start_pos, PREFILL,
                        PREFILL, workspace=aws)
    attp()
    ms = time_events(attp, 2 * L)
    flops = 4.0 * m.heads_local * m.head_dim * PREFILL * (PREFILL + 1) / 2
    byts = 2 * PREFILL * m.kv_heads_local * m.head_dim * 2 + 2 * 2 * PREFILL * m.heads_local * m.head_dim
    res["attn_prefill"] = {"ms": ms, "tflops": flops / ms / 1e9, "flops": flops, "bytes": byts,
                           "gbs": byts / ms / 1e6}
    return res


def parity_check(m, g, w):
    """The timed path against the eager one on the bench's own inputs: one
    more graph replay (StepGraph.run) and one forward_batch on the same host
    inputs (every rank takes part under TP). Greedy tokens must agree except
    where the eager logits' own gap is a near-tie (2^-7 * |top|), and the
    logits within 1e-2 of their range."""
    import numpy as np
    import torch

    tok_g = g.run(w["ids"], w["start_pos"], w["tables"])
    lg_g = m.gather_logits(g.logits).float()
    lg_e, tok_e = m.forward_batch(w["ids"], w["q_lens"], w["start_pos"], w["tables"])
    lg_e = lg_e.float()
    torch.cuda.synchronize()
    err = float((lg_g - lg_e).abs().max() / lg_e.abs().max().clamp_min(1e-30))
    tok_e = tok_e.cpu().numpy()
    diff = np.nonzero(tok_g != tok_e)[0].tolist()
    top = lg_e.max(dim=1).values
    ties = [i for i in diff if float(top[i] - lg_e[i, int(tok_g[i])]) <= 2.0 ** -7 * abs(float(top[i]))]
    return {"graph_vs_forward_batch_logits_rel_err": err, "tokens_compared": int(len(tok_g)),
            "tokens_differing": len(diff), "near_tie_differences": len(ties),
            "parity_ok": bool(err < 1e-2 and len(ties) == len(diff))}


def tp_reduce_timing(m, T, iters=8):
    """Per-call device time of one row-parallel linear + reduction + RMSNorm
    (the o_proj position of layer 0, T tokens) on the model's transport, and
    of the same linear + RMSNorm with no exchange; CUDA-graph replay, max
    over ranks. Every rank calls it."""
    import torch
    import torch.distributed as dist

    from pageserve_b200.model import rms_norm_fused

    dev = m.device
    fl = m.fused[0]
    x = torch.randn(T, m.heads_local * m.head_dim, device=dev, dtype=m.dtype)
    xr = torch.randn(T, m.hidden_size, device=dev, dtype=m.dtype)
    eps = m.rms_eps
    comm = m.comm
    state = {"i": 0, "old": xr}

    def exchange():
        s_ = state["i"] & 1  # the sets alternate as o_proj / down_proj do
        state["i"] += 1
        if m.tp_comm == "fused2":
            comm.linear_push(x, fl.o, s_, workspace=m.lin_ws, scatter=True)
            comm.reduce_norm(state["old"], fl.post_ln, eps, s_, T)
            state["old"] = comm.gathered_ptr(s_)
        elif m.tp_comm == "fused":
            comm.linear_push(x, fl.o, s_, workspace=m.lin_ws)
            comm.allreduce_rmsnorm(xr, fl.post_ln, eps, s_)
        else:
            y = m._linear(x, fl.o, residual=xr if m.tp.rank == 0 else None)
            m.tp.all_reduce_(y)
            rms_norm_fused(y, fl.post_ln, eps)

    def local():
        y = m._linear(x, fl.o, residual=xr)
        rms_norm_fused(y, fl.post_ln, eps)

    out = {}
    for name, fn in (("linear_reduce_norm_us", exchange), ("linear_norm_alone_us", local)):
        dist.barrier()
        torch.cuda.synchronize()
        ms = time_events(fn, iters)
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[name] = round(t.item() * 1e3, 2)
    out["exchange_us"] = round(out["linear_reduce_norm_us"] - out["linear_norm_alone_us"], 2)
    out["calls_per_step"] = 2 * len(m.fused)
    out["tokens"] = T
    return out


class ReferenceSampler:
    """The reference algorithm on the host cores: the oracle port of
    engine/model.py:149-193 (numpy/BLAS; every call dequantizes every int8
    weight like QuantizedWeight.get(), engine/quantization.py:40-41), driven
    one sequence per forward_step as engine/runner.py:65-79 does.

    One sample = one decode token of one sequence at the workload's context
    through ``layers`` decoder layers + the embedding, final norm and lm_head;
    every decode sequence of the workload costs the same. The full-depth time
    per token is the measured per-layer time x the model's layer count + the
    measured head time (decoder layers are identical in cost)."""

    def __init__(self, layers: int, seed: int = 0):
        import numpy as np

        from oracle.model import OracleCausalLM
        from pageserve_b200 import synthetic

        self.full = synthetic.SHAPES[SHAPE_NAME]
        self.layers = max(1, min(layers, self.full.num_layers))
        shape = self.full.with_layers(self.layers)
        sd = synthetic.generate_state_dict(shape, seed=seed)
        self.o = OracleCausalLM(sd, shape, quantize=True, max_position=max(4096, CTX))
        del sd
        nb = CTX // BLOCK + 2
        self.o.allocate_kv_cache(nb, BLOCK)
        rng = np.random.default_rng(seed + 1)
        self.o.k_cache[:] = rng.standard_normal(self.o.k_cache.shape, dtype=np.float32)
        self.o.v_cache[:] = self.o.k_cache
        self.table = list(range(nb))
        self.rng = rng

    def step(self):
        """(wall seconds of the sample, estimated full-depth seconds per decode token)"""
        t = {}
        t0 = time.perf_counter()
        self.o.forward_step([int(self.rng.integers(0, self.full.vocab))], self.table, CTX - 1, timings=t)
        wall = time.perf_counter() - t0
        return wall, t["layers"] / self.layers * self.full.num_layers + t["head"]

    def sample_text(self):
        return (f"oracle port of the reference step (numpy/BLAS, per-sequence forward_step, per-call dequant): "
                f"one decode token of one sequence at context {CTX} per step through {self.layers} of "
                f"{self.full.num_layers} layers + head, per-layer time scaled to the full depth; the prefill "
                f"chunk's share is not charged to the reference (its tok/s is lower by that share)")


def _reference_layers(n_steps: int, budget_s: float = 60.0, cap: int = 8) -> int:
    """Sampled layers (at most `cap`: building the random-init layers costs
    several seconds each) so that n_steps samples take about budget_s (the
    port spends ~0.15-0.3 s per 77 M int8 weights of a layer and per 0.3 G
    lm_head elements on 8-16 host cores)."""
    sh = _shape()
    H, D, I = sh.hidden, sh.head_dim, sh.intermediate
    per_layer_params = H * (sh.num_heads + 2 * sh.num_kv_heads) * D + sh.num_heads * D * H + 3 * H * I
    per_layer_s = 0.3 * per_layer_params / 77e6
    head_s = 0.3 * sh.vocab * H / 0.31e9
    per_step = budget_s / max(1, n_steps)
    return max(1, min(cap, sh.num_layers, int((per_step - head_s) / per_layer_s)))


def cpu_baseline_sample(steps: int = 3):
    """The reference arm's measurement, small (rank 0, N = 1): a few samples
    of ReferenceSampler; tok/s of the full-depth estimate."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    smp = ReferenceSampler(_reference_layers(steps + 1, budget_s=25.0))
    smp.step()
    ests = [smp.step()[1] for _ in range(steps)]
    est = statistics.median(ests)
    return {"value": 1.0 / est, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": smp.sample_text()}


# ------------------------------------------------------------------ run ----

def run_reference(args):
    """--impl reference: the reference's algorithm on the host cores (the
    oracle port: the reference is pure Python/torch without a build, and it
    is not present on the GPU box). Rank 0 alone works; K steps of one
    ReferenceSampler sample each, timed on the host clock."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    smp = ReferenceSampler(_reference_layers(args.steps + args.warmup))
    for _ in range(args.warmup):
        smp.step()
    walls, ests = [], []
    for _ in range(args.steps):
        wall, est = smp.step()
        walls.append(wall)
        ests.append(est)
    v = 1.0 / statistics.median(ests)
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(walls), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random init)",
            "config": _config({"parallelism": "host CPU"}), "impl": "reference",
            "step_definition": "one sample: one decode token of one sequence, "
                               f"{smp.layers} of {smp.full.num_layers} layers (ms_per_step is its wall time)",
            "full_depth_ms_per_token": 1e3 * statistics.median(ests),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": smp.sample_text()},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    from pageserve_b200 import _lib
    from pageserve_b200.model import StepGraph
    from pageserve_b200.tensor_parallel import TPGroup

    peaks = _peaks()
    tp = TPGroup.from_default() if (world > 1 and not args.replicas) else None
    m, w = build_workload(device, seed=0 if tp else rank, tp=tp, tp_comm=args.tp_comm)
    max_blocks = max(len(t) for t in w["tables"])
    g = StepGraph(m, w["q_lens"], max_blocks, CTX, w["start_pos"], w["tables"], w["ids"])
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    # The clock sampler starts (and waits for its first sample, 0.1-1 s, a
    # different time on every rank) before the barrier: with it between the
    # barrier and the start event, the first collective of the early ranks
    # waited for the late ones inside their timed window (N > 1 read slower
    # than end to end).
    with Clocks(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        start.record()
        for _ in range(args.steps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = start.elapsed_time(end)
    if world > 1:
        dist.barrier()
    launches = g.launches_per_replay * args.steps + (_lib.launch_count() - launches0)
    # e2e: host inputs -> public step API -> host next tokens
    for _ in range(2):
        g.run(w["ids"], w["start_pos"], w["tables"])
    torch.cuda.synchronize()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        g.run(w["ids"], w["start_pos"], w["tables"])
    e_end.record()
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_end)
    _lib.raise_on_device_error()
    if world > 1:
        t = torch.tensor([ms, e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e_ms = t.tolist()
    parity = parity_check(m, g, w)
    tp_red = tp_reduce_timing(m, sum(w["q_lens"])) if tp else None
    _lib.raise_on_device_error()
    jobs = 1 if tp else world  # TP: one model over all ranks; replicas: one model per rank
    value = jobs * N_DECODE * args.steps / (ms / 1e3)
    e2e = jobs * N_DECODE * args.steps / (e_ms / 1e3)
    kb = kernel_breakdown(m, w, peaks) if (rank == 0 and not args.no_breakdown) else None
    if world > 1:
        dist.barrier()
    if rank != 0:
        _finish(g, m, world)
        return
    if kb is None:
        print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "ms_per_step": ms / args.steps,
                          "e2e": e2e, "parity": parity, **({"tp_reduce": tp_red} if tp_red else {}),
                          "note": "no per-kernel breakdown"}), flush=True)
        _finish(g, m, world)
        return
    # dominant kernel: the largest per-step time share among the measured classes
    per_step = {k: v["ms"] * (len(m.fused) if k in ("qkv", "o_proj", "gate_up", "down", "attn_decode", "attn_prefill") else 1)
                for k, v in kb.items()}
    dom = max(per_step, key=per_step.get)
    d = kb[dom]
    tensor_bound = dom in ("qkv", "o_proj", "gate_up", "down", "attn_prefill") and \
        d["flops"] / peaks["bf16_tflops"] / 1e12 > \
        d["bytes"] / peaks["hbm_gbs"] / 1e9
    traffic, traffic_src = profile_traffic(dom)
    if tensor_bound:
        roof = {"kernel": dom, "bound": "tensor", "achieved": d["tflops"], "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": d["tflops"] / peaks["bf16_tflops"], "traffic": traffic,
                "algorithmic_per_launch": d["flops"], "algorithmic_bytes_per_launch": d["bytes"],
                "peak_source": peaks["source"] + " (burst)", "traffic_source": traffic_src}
    else:
        roof = {"kernel": dom, "bound": "hbm", "achieved": d["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": d["gbs"] / peaks["hbm_gbs"], "traffic": traffic, "algorithmic_per_launch": d["bytes"],
                "peak_source": peaks["source"], "traffic_source": traffic_src}
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        cpu = cpu_baseline_sample()
    clocks = clk.summary()
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random init, random KV contents)",
            "config": _config({"parallelism": (f"tp{world}" if tp else f"replicas x{world}") if world > 1
                               else "single GPU",
                               **({"tp_allreduce": TP_COMM_NAMES[m.tp_comm]} if tp else {})}),
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": g.h2d_bytes, "d2h_bytes_per_step": g.d2h_bytes,
                    "api": "StepGraph.run (host ids/metadata in, host next tokens out)"},
            "gpu_launches": launches, "launches_per_step": g.launches_per_replay,
            "parity": parity, **({"tp_reduce": tp_red} if tp_red else {}),
            "roofline": roof,
            "kernels": {k: {kk: (round(vv, 4) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                        for k, v in kb.items()},
            "cpu_baseline": None if cpu is None else {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "clocks": clocks, "hbm_peak_gb_rank0": round(torch.cuda.max_memory_allocated(device) / 1e9, 2)}
    print(json.dumps(line), flush=True)
    _finish(g, m, world)


def _finish(g, m, world):
    """Release the CUDA graph (it may hold NCCL calls) and the fused
    all-reduce's IPC mappings on every rank, then leave the process group."""
    import torch.distributed as dist
    g.release()
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="pageserve_b200", choices=["pageserve_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-breakdown", action="store_true", help="skip the per-kernel timing (for profiling runs)")
    ap.add_argument("--replicas", action="store_true", help="N>1: independent replicas instead of tensor parallelism")
    ap.add_argument("--prefill", type=int, default=None,
                    help="prefill chunk tokens per step (default 512 = BASELINE config 4; 0 = decode-only step)")
    ap.add_argument("--tp-comm", default="auto", choices=["auto", "fused", "fused2", "nccl"],
                    help="N>1 tensor parallelism: row-parallel reduction transport")
    ap.add_argument("--config", type=int, default=4, choices=[4, 5],
                    help="BASELINE configuration: 4 = 3B-shape mixed step (default), 5 = 32B-shape TP decode")
    args = ap.parse_args()
    global PREFILL
    if args.config == 5:
        _use_config5()
    if args.prefill is not None:
        PREFILL = max(0, args.prefill)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
