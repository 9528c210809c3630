"""Host logic of the fused tensor-parallel all-reduce, on CPU: the receive
buffer layout the C ABI reports, and the IPC handle exchange of
``FusedAllReduce.create`` over 2 gloo ranks with a fake library (no device
calls): every rank ends with its own buffer at its own index and each peer's
buffer opened from that peer's handle."""

import ctypes
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from pageserve_b200 import _lib


def test_buffer_bytes_layout():
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    lib = _lib.load()
    # control words (4 KB) + the gathered residual [2 sets][max_tokens][hidden] (256-byte padded)
    # + slots [2 sets][world][max_tokens][hidden] of 2-byte elements
    assert lib.ps_comm_buffer_bytes(2, 576, 2048, _lib.PS_BF16) == 4096 + 2 * 576 * 2048 * 2 + 2 * 2 * 576 * 2048 * 2
    assert lib.ps_comm_buffer_bytes(8, 1, 8, _lib.PS_F16) == 4096 + 256 + 2 * 8 * 8 * 2
    # the gathered region of set s starts after the control words
    assert lib.ps_comm_gathered_offset(2, 576, 2048, _lib.PS_BF16, 0) == 4096
    assert lib.ps_comm_gathered_offset(2, 576, 2048, _lib.PS_BF16, 1) == 4096 + 576 * 2048 * 2
    assert lib.ps_comm_gathered_offset(2, 576, 2048, _lib.PS_BF16, 2) == 0
    assert lib.ps_comm_buffer_bytes(9, 1, 8, _lib.PS_BF16) == 0  # above PS_COMM_MAX_WORLD
    assert lib.ps_comm_buffer_bytes(2, 1, 8, _lib.PS_F32) == 0   # 16-bit activations only
    assert lib.ps_comm_buffer_bytes(0, 1, 8, _lib.PS_BF16) == 0


class _FakeLib:
    """Stands in for the C library: 'device' buffers are integers, a handle
    encodes (owner rank, buffer) and opening it maps to a distinct address."""

    def __init__(self, rank):
        self.rank = rank
        self.freed, self.closed = [], []

    def ps_comm_buffer_bytes(self, world, max_tokens, hidden, dtype):
        return 1024 + 2 * world * max_tokens * hidden * 2

    def ps_comm_alloc(self, pref, nbytes):
        ctypes.cast(pref, ctypes.POINTER(ctypes.c_void_p))[0] = 0x10000 * (self.rank + 1)
        return 0

    def ps_ipc_get_handle(self, buf, h):
        raw = f"rank{self.rank}:{buf}".encode().ljust(64, b"\0")
        ctypes.memmove(h, raw, 64)
        return 0

    def ps_ipc_open_handle(self, h, pref):
        owner, buf = bytes(h).rstrip(b"\0").decode().split(":")
        assert owner != f"rank{self.rank}", "a rank never opens its own handle"
        ctypes.cast(pref, ctypes.POINTER(ctypes.c_void_p))[0] = 0x7000000 + int(buf)
        return 0

    def ps_ipc_close(self, p):
        self.closed.append(p)
        return 0

    def ps_comm_free(self, p):
        self.freed.append(p)
        return 0


def _worker(rank, world, sync_file, out_file):
    import torch.distributed as dist

    from pageserve_b200 import comm
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"file://{sync_file}")
    fake = _FakeLib(rank)
    _lib.load = lambda: fake  # noqa: E731  (this child process only)
    torch.cuda.set_device = lambda d: None  # no device on the CPU runner
    ar = comm.FusedAllReduce.create(rank, world, 16, 64, torch.bfloat16, "cpu")
    bufs = [ar._rank_bufs[r] for r in range(world)]
    torch.cuda.synchronize = lambda d=None: None
    ar.close()
    torch.save({"bufs": bufs, "own": ar.buf, "freed": fake.freed, "closed": fake.closed}, f"{out_file}.{rank}")
    dist.destroy_process_group()


def test_handle_exchange_two_ranks():
    world = 2
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_worker, args=(world, os.path.join(tmp, "sync"), os.path.join(tmp, "out")), nprocs=world, join=True)
        res = [torch.load(os.path.join(tmp, f"out.{r}"), weights_only=True) for r in range(world)]
    for r in range(world):
        own = 0x10000 * (r + 1)
        assert res[r]["own"] == own
        assert res[r]["bufs"][r] == own
        for p in range(world):
            if p != r:
                assert res[r]["bufs"][p] == 0x7000000 + 0x10000 * (p + 1)  # opened from rank p's handle
        assert res[r]["freed"] == [own]
        assert sorted(res[r]["closed"]) == sorted(b for i, b in enumerate(res[r]["bufs"]) if i != r)


def test_auto_tp_transport_choice():
    """tp_comm="auto": the one-shot push at 2 ranks, NCCL from 4 (measured);
    the two-shot transport needs 128-column slices."""
    from pageserve_b200.model import auto_tp_comm, two_shot_ok
    assert auto_tp_comm(2, 2048) == "fused"
    assert auto_tp_comm(4, 2048) == "nccl" and auto_tp_comm(8, 5120) == "nccl"
    assert two_shot_ok(8, 2048) and two_shot_ok(4, 5120) and two_shot_ok(2, 256)
    assert not two_shot_ok(8, 896) and not two_shot_ok(1, 2048) and not two_shot_ok(3, 2048)
