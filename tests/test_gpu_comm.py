"""The fused tensor-parallel all-reduce kernels (ps_linear_push +
ps_allreduce_rmsnorm) on one GPU, with W ranks emulated in one process:
every rank's push is issued before any rank's consume of the same set, so
no kernel waits for a later launch. Checked against the unfused path:
per-rank partials from the plain W8A16/16-bit linear (engine/
tensor_parallel.py:34-46), summed in rank order (the all-reduce,
tensor_parallel.py:47), then the residual add and RMSNorm of
engine/model.py:184-190."""

import pytest
import torch

from pageserve_b200 import _lib
from pageserve_b200.comm import FusedAllReduce
from pageserve_b200.model import rms_norm_fused
from pageserve_b200.quantization import QuantizedWeight, linear16

pytestmark = pytest.mark.gpu

REL_TOL = 2e-2  # bf16 output of a different reduction order (the RMSNorm)


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def rel_err(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _partial(x, w):
    if isinstance(w, QuantizedWeight):
        return w.linear(x)
    return linear16(x, w)


def _weights(world, N, K, int8, dev, g):
    ws = []
    for _ in range(world):
        w = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        ws.append(QuantizedWeight(w) if int8 else w)
    return ws


@pytest.mark.parametrize("world,M,N,K,int8", [
    (2, 576, 2048, 1024, True),    # TP2 o_proj of the 3B shape, prefill+decode batch (split-K writer)
    (2, 64, 2048, 5504, True),     # TP2 down_proj, decode batch
    (4, 96, 1024, 256, True),      # 4 K tiles: no split, the GEMM epilogue pushes
    (2, 40, 512, 640, False),      # 16-bit weight (SS operands)
    (1, 33, 256, 512, True),       # degenerate world of one
    (8, 17, 2048, 256, True),      # TP8 o_proj width
    (2, 9, 1024, 512, True),       # decode-sized: the mma.sync small-M linear pushes
    (2, 4, 1024, 8192, True),      # decode-sized, long K: the cp.async-ring small-M linear pushes
])
def test_push_then_allreduce_rmsnorm(world, M, N, K, int8):
    _need_gpu()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(world * 1000 + M)
    ranks = FusedAllReduce.emulated(world, max_tokens=max(M, 64), hidden=N, dtype=torch.bfloat16, device=dev)
    try:
        xs = [torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16) for _ in range(world)]
        ws = _weights(world, N, K, int8, dev, g)
        norm_w = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(torch.bfloat16)
        resid = [torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16) for _ in range(world)]
        resid = [resid[0].clone() for _ in range(world)]  # every rank holds the same residual stream
        partials = [_partial(xs[r], ws[r]) for r in range(world)]
        s = torch.zeros(M, N, dtype=torch.float32, device=dev)
        for p in partials:
            s += p.float()
        s = s.to(torch.bfloat16)
        x_ref = (resid[0].float() + s.float()).to(torch.bfloat16)
        y_ref = rms_norm_fused(x_ref, norm_w, 1e-6)
        # three rounds over both sets: the flags re-arm
        for it in range(3):
            for set_ in (0, 1):
                for r in range(world):
                    ranks[r].linear_push(xs[r], ws[r], set_)
                if set_ == 0:
                    xr = [resid[r].clone() for r in range(world)]
                    ys = [ranks[r].allreduce_rmsnorm(xr[r], norm_w, 1e-6, set_) for r in range(world)]
                    torch.cuda.synchronize()
                    for r in range(world):
                        assert torch.equal(xr[r], x_ref), f"round {it} rank {r}: residual stream"
                        assert torch.equal(ys[r], ys[0]), f"round {it}: ranks disagree"
                    assert rel_err(ys[0].float(), y_ref.float()) < REL_TOL
                else:
                    outs = [ranks[r].allreduce_rmsnorm(None, None, 0.0, set_, M=M) for r in range(world)]
                    torch.cuda.synchronize()
                    for r in range(world):
                        assert torch.equal(outs[r], s), f"round {it} rank {r}: plain all-reduce"
        _lib.raise_on_device_error()
    finally:
        ranks[0].close()


@pytest.mark.parametrize("world,M,N,K,int8", [
    (2, 576, 2048, 1024, True),    # TP2 o_proj of the 3B shape (split-K writer)
    (4, 576, 2048, 512, True),     # TP4 o_proj, prefill+decode batch
    (8, 576, 2048, 256, True),     # TP8 o_proj: 256-column slices
    (8, 9, 2048, 1376, True),      # TP8 down_proj at decode size (mma.sync small-M writer)
    (4, 128, 5120, 1280, True),    # 32B shape TP4 o_proj, config-5 batch
    (2, 40, 512, 640, False),      # 16-bit weight
])
def test_two_shot_scatter_reduce_gather_rmsnorm(world, M, N, K, int8):
    """Two-shot form: ps_linear_push_scatter sends each column slice to its
    owner rank, ps_tp_reduce_rmsnorm (phase 1 on every rank, then phase 2 on
    every rank: no kernel waits on a later launch) reduces the slice, adds the
    residual, all-gathers it and normalises. The gathered residual stream is
    bit-exact (the same partials and rank order as the unfused sum), identical
    on every rank, and feeds the next set's reduction as its x_old; rounds
    alternate the sets, so the flags and row-block counters re-arm."""
    _need_gpu()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(world * 77 + M)
    ranks = FusedAllReduce.emulated(world, max_tokens=max(M, 64), hidden=N, dtype=torch.bfloat16, device=dev)
    try:
        xs = [torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16) for _ in range(world)]
        ws = _weights(world, N, K, int8, dev, g)
        norm_w = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(torch.bfloat16)
        resid = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
        partials = [_partial(xs[r], ws[r]) for r in range(world)]
        s = torch.zeros(M, N, dtype=torch.float32, device=dev)
        for p in partials:
            s += p.float()
        s = s.to(torch.bfloat16)
        x_exp = resid
        x_old = [resid] * world
        for it in range(3):
            for set_ in (0, 1):
                for r in range(world):
                    ranks[r].linear_push(xs[r], ws[r], set_, scatter=True)
                for r in range(world):
                    ranks[r].reduce_norm(x_old[r], norm_w, 1e-6, set_, M, phases=1)
                ys = [ranks[r].reduce_norm(x_old[r], norm_w, 1e-6, set_, M, phases=2) for r in range(world)]
                torch.cuda.synchronize()
                x_exp = (x_exp.float() + s.float()).to(torch.bfloat16)
                y_ref = rms_norm_fused(x_exp, norm_w, 1e-6)
                for r in range(world):
                    assert torch.equal(ranks[r].gathered(set_, M), x_exp), f"round {it} set {set_} rank {r}: residual"
                    assert torch.equal(ys[r], ys[0]), f"round {it} set {set_}: ranks disagree"
                assert rel_err(ys[0].float(), y_ref.float()) < REL_TOL
                x_old = [ranks[r].gathered_ptr(set_) for r in range(world)]
        # the plain all-reduce (no residual, no norm): y = T(sum of partials)
        for r in range(world):
            ranks[r].linear_push(xs[r], ws[r], 0, scatter=True)
        for r in range(world):
            ranks[r].reduce_norm(None, None, 0.0, 0, M, phases=1)
        outs = [ranks[r].reduce_norm(None, None, 0.0, 0, M, phases=2) for r in range(world)]
        torch.cuda.synchronize()
        for r in range(world):
            assert torch.equal(outs[r], s), f"rank {r}: plain two-shot all-reduce"
        _lib.raise_on_device_error()
    finally:
        ranks[0].close()


def test_row_parallel_linear_on_push_transport_matches_oracle():
    """tensor_parallel.py:34-48 semantics (the sum of the ranks' partials of
    a column-split weight) against the numpy oracle."""
    _need_gpu()
    from oracle import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    world, M, N, K = 2, 48, 768, 1024
    w = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    q, sc = ops.quantize_per_channel(w.float().cpu().numpy())
    xn = x.float().cpu().numpy()
    shards = [slice(r * K // world, (r + 1) * K // world) for r in range(world)]
    ref = ops.round_bf16(sum(ops.round_bf16(ops.quantized_linear(xn[:, sl], q[:, sl], sc)) for sl in shards))
    full = QuantizedWeight(w)
    ranks = FusedAllReduce.emulated(world, max_tokens=M, hidden=N, dtype=torch.bfloat16, device=dev)
    try:
        shards = []
        for r in range(world):
            sl = slice(r * K // world, (r + 1) * K // world)
            shards.append(QuantizedWeight.from_quantized(full.q[:, sl].contiguous(), full.scale, torch.bfloat16))
        for r in range(world):
            ranks[r].linear_push(x[:, r * K // world:(r + 1) * K // world].contiguous(), shards[r], 0)
        outs = [ranks[r].allreduce_rmsnorm(None, None, 0.0, 0, M=M) for r in range(world)]
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1])
        assert rel_err(outs[0].float().cpu(), torch.from_numpy(ref).float()) < REL_TOL
    finally:
        ranks[0].close()


def test_consumer_wait_times_out_without_producer():
    """A flag that nothing raises: the bounded wait gives up (a few
    seconds), records the timeout in the device status word, and the
    context stays usable."""
    _need_gpu()
    dev = torch.device("cuda", 0)
    (rank,) = FusedAllReduce.emulated(1, max_tokens=8, hidden=256, dtype=torch.bfloat16, device=dev)
    try:
        _lib.raise_on_device_error()  # nothing pending from earlier tests
        x = torch.zeros(4, 256, dtype=torch.bfloat16, device=dev)
        w = torch.ones(256, dtype=torch.bfloat16, device=dev)
        rank.allreduce_rmsnorm(x, w, 1e-6, 1)
        torch.cuda.synchronize()
        assert _lib.device_status(clear=True) == 4  # kErrTimeout
        # the buffer is marked broken: the next wait gives up at once
        rank.allreduce_rmsnorm(x, w, 1e-6, 0)
        torch.cuda.synchronize()
        assert _lib.device_status(clear=True) == 4
        rank.reset()
        # still usable after re-zeroing: a normal push/consume round
        xin = torch.randn(4, 64, device=dev).to(torch.bfloat16)
        wt = (torch.randn(256, 64, device=dev) * 0.1).to(torch.bfloat16)
        rank.linear_push(xin, wt, 1)
        out = rank.allreduce_rmsnorm(None, None, 0.0, 1, M=4)
        torch.cuda.synchronize()
        assert torch.equal(out, linear16(xin, wt))
        _lib.raise_on_device_error()
    finally:
        rank.close()
