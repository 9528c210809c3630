"""Kernel microbenchmarks (BASELINE configs 2 and 3) and small profiling cases.

    python -m pageserve_b200.microbench linear --M 576 --N 22016 --K 2048
    python -m pageserve_b200.microbench sweep          # config 3: W8A16 sweep
    python -m pageserve_b200.microbench attn           # config 2: paged decode attention

Timing: the timed launches are captured once into a CUDA graph and the graph
is replayed between CUDA events (device time without host launch overhead —
the way the model step runs); the weight (or KV cache) is replicated over
enough copies that the rotation exceeds the 126 MB L2, so every launch
streams from HBM. Prints one JSON object per case.
"""

from __future__ import annotations

import argparse
import json
import math
import sys

import numpy as np
import torch

L2_BYTES = 126 * 2 ** 20


def _peaks():
    import json as _j
    from pathlib import Path
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if p.exists():
        d = _j.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"]
    return 6650.0, 1590.0


def _time(fn, iters, warmup=3, graph=True):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    if not graph:
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / iters
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_linear(M, N, K, iters=20, seed=0, bf16_weight=False, warmup=3, tiled=True, swiglu=False):
    """swiglu: N = 2I rows (interleaved gate/up) through ps_linear_swiglu,
    output (M, I) — the step's gate|up projection."""
    from .quantization import (LinearWorkspace, QuantizedWeight, linear16, linear_swiglu, tile_int8_weight,
                               w8a16_linear)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    wbytes = N * K * (2 if bf16_weight else 1)
    copies = max(1, math.ceil(2 * L2_BYTES / wbytes)) if iters > 1 else 1
    if bf16_weight:
        ws = [torch.randn(N, K, device=dev, generator=g, dtype=torch.bfloat16) for _ in range(copies)]
    else:
        ws = [torch.randint(-127, 128, (N, K), device=dev, generator=g, dtype=torch.int8) for _ in range(copies)]
        tws = [tile_int8_weight(w) for w in ws] if tiled else [None] * copies
    scale = torch.empty(N, 1, device=dev).uniform_(1e-3, 1e-2, generator=g)
    x = torch.randn(M, K, device=dev, generator=g, dtype=torch.bfloat16)
    out = torch.empty(M, N // 2 if swiglu else N, device=dev, dtype=torch.bfloat16)
    wsp = LinearWorkspace()
    ctr = [0]
    qws = [QuantizedWeight.from_quantized(w, scale, torch.bfloat16) for w in ws] if (swiglu and not bf16_weight) \
        else None
    for qw in qws or []:
        qw.tiled()  # build every tiled copy before the timed graph is captured

    def f():
        w = ws[ctr[0] % copies]
        ctr[0] += 1
        if swiglu:
            linear_swiglu(x, w if bf16_weight else qws[(ctr[0] - 1) % copies], out=out)
        elif bf16_weight:
            linear16(x, w, out=out, workspace=wsp)
        else:
            w8a16_linear(x, w, scale, out=out, workspace=wsp, q_tiled=tws[(ctr[0] - 1) % copies])
    ms = _time(f, iters, warmup)
    hbm, tf = _peaks()
    flops = 2.0 * M * N * K
    byts = wbytes + (0 if bf16_weight else 4 * N) + 2 * M * K + 2 * M * (N // 2 if swiglu else N)
    bound = "tensor" if flops / (tf * 1e12) > byts / (hbm * 1e9) else "hbm"
    ach_tf = flops / ms / 1e9
    ach_gb = byts / ms / 1e6
    return {"case": "linear_swiglu" if swiglu else "linear", "M": M, "N": N, "K": K,
            "weight": "bf16" if bf16_weight else "int8",
            "layout": "tiled" if (tiled and not bf16_weight) else "row-major", "us": ms * 1e3,
            "tflops": ach_tf, "gbs": ach_gb, "bound": bound,
            "frac": (ach_tf / tf) if bound == "tensor" else (ach_gb / hbm),
            "ideal_us": max(flops / (tf * 1e12), byts / (hbm * 1e9)) * 1e6}


def bench_attn(B=64, lo=512, hi=4096, Hq=16, Hkv=2, D=128, bs=16, pool=20000, iters=20, seed=0, warmup=3):
    """paged decode attention, bf16, ctx ~ U[lo, hi],
    block tables a random permutation of a 20k-block pool."""
    from .paged_attention import AttentionWorkspace, paged_attention
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(lo, hi + 1, (B,), generator=g)
    nblk = [(int(c) + bs - 1) // bs for c in ctx]
    assert sum(nblk) <= pool
    perm = torch.randperm(pool, generator=g)
    mb = max(nblk)
    tab = torch.full((B, mb), -1, dtype=torch.int32)
    at = 0
    for b, n in enumerate(nblk):
        tab[b, :n] = perm[at:at + n].to(torch.int32)
        at += n
    kv_bytes = pool * bs * Hkv * D * 2
    copies = max(1, math.ceil(2 * L2_BYTES / (2 * kv_bytes))) if iters > 1 else 1
    gd = torch.Generator(device=dev)
    gd.manual_seed(seed)
    caches = [(torch.randn(pool, bs, Hkv, D, device=dev, generator=gd, dtype=torch.bfloat16),
               torch.randn(pool, bs, Hkv, D, device=dev, generator=gd, dtype=torch.bfloat16)) for _ in range(copies)]
    q = torch.randn(B, Hq, D, device=dev, generator=gd, dtype=torch.bfloat16)
    tab = tab.to(dev)
    cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
    sp = (ctx - 1).to(torch.int32).to(dev)
    out = torch.empty_like(q)
    aws = AttentionWorkspace()
    ctr = [0]

    def f():
        kc, vc = caches[ctr[0] % copies]
        ctr[0] += 1
        paged_attention(q, kc, vc, tab, cu, sp, 1, int(ctx.max()), out=out, workspace=aws)
    ms = _time(f, iters, warmup)
    hbm, _ = _peaks()
    tot = int(ctx.sum())
    byts = tot * Hkv * D * 2 * 2 + 2 * B * Hq * D * 2 + 4 * sum(nblk)
    return {"case": "attn_decode", "B": B, "ctx_sum": tot, "us": ms * 1e3, "bytes": byts, "gbs": byts / ms / 1e6,
            "frac": byts / ms / 1e6 / hbm, "ideal_us": byts / (hbm * 1e9) * 1e6}


def bench_attn_prefill(T=512, start=0, Hq=16, Hkv=2, D=128, bs=16, iters=20, seed=0, warmup=3):
    """One causal prefill chunk of T tokens at ``start`` (the config-4 chunk)."""
    from .paged_attention import AttentionWorkspace, paged_attention
    dev = torch.device("cuda")
    ctx = start + T
    nblk = (ctx + bs - 1) // bs
    pool = max(4 * nblk, 64)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    kc = torch.randn(pool, bs, Hkv, D, device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(pool, bs, Hkv, D, device=dev, generator=g, dtype=torch.bfloat16)
    q = torch.randn(T, Hq, D, device=dev, generator=g, dtype=torch.bfloat16)
    tab = torch.randperm(pool, device=dev)[:nblk].to(torch.int32).reshape(1, -1)
    cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
    sp = torch.tensor([start], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    aws = AttentionWorkspace()
    ms = _time(lambda: paged_attention(q, kc, vc, tab, cu, sp, T, ctx, out=out, workspace=aws), iters, warmup)
    flops = 4.0 * Hq * D * sum(start + i + 1 for i in range(T))
    return {"case": "attn_prefill", "T": T, "start": start, "us": ms * 1e3, "tflops": flops / ms / 1e9}


def bench_tp_reduce(M=576, H=2048, K_full=2048, iters=20, warmup=3, seed=0):
    """Row-parallel linear + all-reduce + RMSNorm of one layer position under
    tensor parallelism (run under torchrun, one rank per GPU): NCCL all_reduce
    vs the fused peer-memory push, vs the linear + norm alone (no exchange).
    Device time per iteration, max over ranks."""
    import torch.distributed as dist

    from .comm import FusedAllReduce
    from .model import rms_norm_fused
    from .quantization import LinearWorkspace, QuantizedWeight
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(seed + rank)
    K = K_full // world
    w = QuantizedWeight((torch.randn(H, K, device=dev, generator=g) * 0.02).to(torch.bfloat16))
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    resid = torch.randn(M, H, device=dev, generator=torch.Generator(device=dev).manual_seed(seed)).to(torch.bfloat16)
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    ws = LinearWorkspace()
    comm = FusedAllReduce.create(rank, world, M, H, torch.bfloat16, dev)
    xr = resid.clone()

    def nccl():
        y = w.linear(x, residual=xr if rank == 0 else None, workspace=ws)
        dist.all_reduce(y)
        rms_norm_fused(y, nw, 1e-6)

    it = [0]

    def fused():  # the sets must alternate, as o_proj / down_proj do in a layer
        s_ = it[0] & 1
        it[0] += 1
        comm.linear_push(x, w, s_, workspace=ws)
        comm.allreduce_rmsnorm(xr, nw, 1e-6, s_)

    two_shot = H % world == 0 and (H // world) % 128 == 0 and world > 1
    it2 = [0]
    x_old = [xr]

    def fused2():  # two-shot: scatter, reduce + all-gather, local norm; sets alternate
        s_ = it2[0] & 1
        it2[0] += 1
        comm.linear_push(x, w, s_, workspace=ws, scatter=True)
        comm.reduce_norm(x_old[0], nw, 1e-6, s_, M)
        x_old[0] = comm.gathered_ptr(s_)

    def local():
        y = w.linear(x, residual=xr, workspace=ws)
        rms_norm_fused(y, nw, 1e-6)

    def push_only():  # producer side alone (flags only accumulate; nothing waits)
        comm.linear_push(x, w, 0, workspace=ws)

    def linear_only():
        w.linear(x, workspace=ws)

    def allreduce_only():
        dist.all_reduce(xr)

    out = {"case": "tp_reduce", "world": world, "M": M, "H": H, "K_shard": K}
    cases = [("nccl_us", nccl), ("fused_us", fused)] + ([("fused2_us", fused2)] if two_shot else []) + \
        [("local_us", local), ("push_only_us", push_only), ("linear_only_us", linear_only),
         ("nccl_allreduce_only_us", allreduce_only)]
    for name, fn in cases:
        dist.barrier()
        ms = _time(fn, iters, warmup)
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[name] = t.item() * 1e3
    torch.cuda.synchronize()
    dist.barrier()
    comm.close()
    return out


SWEEP_NK = [(2560, 2048), (2048, 2048), (22016, 2048), (2048, 11008)]
SWEEP_M = [1, 8, 64, 256, 2048]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["linear", "sweep", "attn", "prefill", "tp"])
    ap.add_argument("--M", type=int, default=576)
    ap.add_argument("--N", type=int, default=22016)
    ap.add_argument("--K", type=int, default=2048)
    ap.add_argument("--bf16-weight", action="store_true")
    ap.add_argument("--row-major", action="store_true", help="int8 weight row-major (2D TMA) instead of pre-tiled")
    ap.add_argument("--swiglu", action="store_true", help="gate|up linear with the SwiGLU epilogue (N = 2I)")
    ap.add_argument("--B", type=int, default=64, help="attn: decode sequences")
    ap.add_argument("--lo", type=int, default=512, help="attn: shortest context")
    ap.add_argument("--hi", type=int, default=4096, help="attn: longest context")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    torch.cuda.init()
    if a.what == "tp":  # under torchrun: one rank per GPU
        import datetime
        import os

        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        for m, kf, h in ((576, 2048, 2048), (576, 11008, 2048), (64, 2048, 2048), (64, 11008, 2048),
                         (128, 5120, 5120), (128, 27648, 5120)):
            r = bench_tp_reduce(M=m, H=h, K_full=kf, iters=a.iters, warmup=a.warmup)
            if dist.get_rank() == 0:
                print(json.dumps(r), flush=True)
        from . import _lib
        _lib.raise_on_device_error()
        dist.barrier()
        dist.destroy_process_group()
        return 0
    if a.what == "linear":
        print(json.dumps(bench_linear(a.M, a.N, a.K, a.iters, bf16_weight=a.bf16_weight, warmup=a.warmup,
                                      tiled=not a.row_major, swiglu=a.swiglu)))
    elif a.what == "sweep":
        for n, k in SWEEP_NK:
            for m in SWEEP_M:
                print(json.dumps(bench_linear(m, n, k, a.iters, warmup=a.warmup, tiled=not a.row_major)), flush=True)
    elif a.what == "prefill":
        print(json.dumps(bench_attn_prefill(iters=a.iters, warmup=a.warmup)))
    else:
        print(json.dumps(bench_attn(B=a.B, lo=a.lo, hi=a.hi, iters=a.iters, warmup=a.warmup)))
    from . import _lib
    _lib.raise_on_device_error()
    return 0


if __name__ == "__main__":
    sys.exit(main())
