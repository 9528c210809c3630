"""Tensor parallelism on 2 GPUs against the oracle.

A TP=2 Megatron-sharded model (engine/tensor_parallel.py:21-48: column-
parallel q|k|v and gate|up, row-parallel o_proj and down_proj followed by a
SUM all-reduce, :47) runs a chunked prefill, then a mixed batch (a chunk at
start_pos 0 plus a decode), with the row-parallel reductions either fused
(peer-memory push into the next RMSNorm) or on NCCL all_reduce. Both ranks'
logits must be identical, within 2e-2 of the numpy oracle's unsharded float32
model (the logit range; engine/model.py:149-193), and their greedy tokens
equal the oracle's except at near-ties (oracle margin <= 2^-7 * |top|). The
TP=1 model is checked against the same oracle values as a control.
Skipped with fewer than 2 GPUs. NVLS stays off (plain peer memory only)."""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _tp_worker(rank, world, port, out_file, tp_comm):
    import datetime

    import torch.distributed as dist

    from pageserve_b200 import _lib, synthetic
    from pageserve_b200.model import PagedCausalLM
    from pageserve_b200.tensor_parallel import TPGroup
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=9, perturb_norms_biases=True)
    m = PagedCausalLM.from_state_dict(sd, shape, device=f"cuda:{rank}", quantize=True, tp=TPGroup(rank, world),
                                      tp_comm=tp_comm, tp_max_tokens=64)
    m.allocate_kv_cache(40, 4)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, shape.vocab, size=n) for n in (11, 23)]
    tables = [list(range(0, 6)), list(range(6, 14))]
    lg0 = m.forward_step(torch.from_numpy(prompts[0]), tables[0], 0)
    lg1, tok = m.forward_batch(np.concatenate([prompts[1][:20], [7]]), [20, 1], [0, 11], [tables[1], tables[0]])
    res = {"lg0": lg0.float().cpu(), "lg1": lg1.float().cpu(), "tok": tok.cpu()}
    if rank == 0:
        ref = PagedCausalLM.from_state_dict(sd, shape, device="cuda:0", quantize=True)
        ref.allocate_kv_cache(40, 4)
        r0 = ref.forward_step(torch.from_numpy(prompts[0]), tables[0], 0)
        r1, rt = ref.forward_batch(np.concatenate([prompts[1][:20], [7]]), [20, 1], [0, 11], [tables[1], tables[0]])
        res.update(ref0=r0.float().cpu(), ref1=r1.float().cpu(), reftok=rt.cpu())
    torch.save(res, f"{out_file}.{rank}")
    _lib.raise_on_device_error()
    m.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("tp_comm,port", [("fused", 29517), ("fused2", 29518), ("nccl", 29519)])
def test_tp2_matches_tp1(tp_comm, port):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_tp_worker, args=(2, port, os.path.join(tmp, "r"), tp_comm), nprocs=2, join=True)
        a = torch.load(os.path.join(tmp, "r.0"), weights_only=True)
        b = torch.load(os.path.join(tmp, "r.1"), weights_only=True)
    for k in ("lg0", "lg1", "tok"):
        assert torch.equal(a[k], b[k]), f"ranks disagree on {k}"
    o0, o1 = _oracle()
    for got, ref in ((a["lg0"], o0), (a["lg1"], o1), (a["ref0"], o0), (a["ref1"], o1)):
        got = got.numpy()
        err = float(np.abs(got - ref).max() / np.abs(ref).max())
        assert err < 2e-2, err
    for toks in (a["tok"], a["reftok"]):
        for i, t in enumerate(toks.tolist()):
            top = float(o1[i].max())
            assert t == int(o1[i].argmax()) or top - o1[i, t] <= 2.0 ** -7 * abs(top), (i, t, int(o1[i].argmax()))


def _oracle():
    """The unsharded float32 oracle on the workers' inputs: logits of the
    prefill (all rows) and of the mixed batch (each sequence's last row)."""
    from oracle.model import OracleCausalLM
    from pageserve_b200 import synthetic
    shape = synthetic.TINY
    sd = synthetic.generate_state_dict(shape, seed=9, perturb_norms_biases=True)
    m = OracleCausalLM(sd, shape, quantize=True)
    m.allocate_kv_cache(40, 4)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, shape.vocab, size=n) for n in (11, 23)]
    tables = [list(range(0, 6)), list(range(6, 14))]
    o0 = m.forward_step(prompts[0], tables[0], 0)
    r1 = m.forward_step(prompts[1][:20], tables[1], 0)[-1]
    r2 = m.forward_step(np.asarray([7]), tables[0], 11)[-1]
    return o0, np.stack([r1, r2])
