"""Fused tensor-parallel all-reduce over peer memory (the B200 replacement of
the ``dist.all_reduce(partial, SUM)`` in engine/tensor_parallel.py:34-48).

Each rank allocates one receive buffer (``ps_comm_alloc``) and maps every
peer's buffer into its own address space through CUDA IPC handles exchanged
with ``torch.distributed`` (one ``all_gather_object`` at setup). Then, per
row-parallel linear:

  ``linear_push(x_shard, weight, set)``   the tensor-core linear whose final
      writer stores its (tokens, hidden) output into slot[rank] of every
      rank's buffer and raises every rank's arrival flag of ``set``;
  ``allreduce_rmsnorm(x, w, eps, set)``   waits for all ranks' slots, sums
      them, adds the residual x (in place) and returns rmsnorm(x) * w —
      or, with ``w=None``, returns the plain reduced sum.

The two slot sets alternate between the o_proj (set 0) and down_proj
(set 1) reductions of a layer. ``FusedAllReduce.emulated`` builds the W
ranks' buffers in one process on one GPU (every rank's kernels issued in
sequence on one stream), which exercises the same kernels and flags
without a second GPU.

Two-shot form (``linear_push(..., scatter=True)`` + ``reduce_norm``): the
linear sends each column slice of its output only to the rank that owns it
(reduce-scatter); the owner sums its slice, adds the residual, and stores the
new residual slice into every rank's gathered region (all-gather), where each
rank normalises whole rows. Per rank that moves 2 (W-1)/W of the output over
NVLink instead of the one-shot's W-1 copies; the residual stream then lives
in the gathered region of the set (``gathered_ptr``).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

HANDLE_BYTES = 64


class FusedAllReduce:
    """One rank's receive buffer plus every rank's buffer as mapped here."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int, dtype: torch.dtype,
                 device: torch.device, own_buf: int, rank_bufs: list[int], opened: list[int]):
        self.rank, self.world = rank, world
        self.max_tokens, self.hidden, self.dtype = max_tokens, hidden, dtype
        self.device = torch.device(device)
        self.buf = own_buf
        self._rank_bufs = (ctypes.c_void_p * world)(*rank_bufs)
        self._opened = opened  # peer mappings to close
        self._owned = [own_buf]  # buffers to free
        self._closed = False

    # ------------------------------------------------------------ setup ----
    @staticmethod
    def buffer_bytes(world: int, max_tokens: int, hidden: int, dtype: torch.dtype) -> int:
        n = _lib.load().ps_comm_buffer_bytes(world, max_tokens, hidden, _lib.dtype_code(dtype))
        if n == 0:
            raise ValueError(f"unsupported fused all-reduce buffer (world={world}, max_tokens={max_tokens}, "
                             f"hidden={hidden}, dtype={dtype})")
        return n

    @staticmethod
    def _alloc(nbytes: int) -> int:
        p = ctypes.c_void_p()
        _lib.check(_lib.load().ps_comm_alloc(ctypes.byref(p), nbytes), "comm_alloc")
        return p.value

    @classmethod
    def create(cls, rank: int, world: int, max_tokens: int, hidden: int, dtype: torch.dtype, device,
               group=None) -> "FusedAllReduce":
        """Collective over ``group`` (every rank calls it): allocate, share
        handles with all_gather_object, open the peers' buffers."""
        import torch.distributed as dist
        lib = _lib.load()
        device = torch.device(device)
        torch.cuda.set_device(device)
        own = cls._alloc(cls.buffer_bytes(world, max_tokens, hidden, dtype))
        h = (ctypes.c_char * HANDLE_BYTES)()
        _lib.check(lib.ps_ipc_get_handle(own, h), "ipc_get_handle")
        handles: list = [None] * world
        dist.all_gather_object(handles, bytes(h), group=group)
        bufs, opened = [], []
        for r, hr in enumerate(handles):
            if r == rank:
                bufs.append(own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_char * HANDLE_BYTES).from_buffer_copy(hr)
            _lib.check(lib.ps_ipc_open_handle(hb, ctypes.byref(p)), "ipc_open_handle")
            bufs.append(p.value)
            opened.append(p.value)
        dist.barrier(group=group)
        return cls(rank, world, max_tokens, hidden, dtype, device, own, bufs, opened)

    @classmethod
    def emulated(cls, world: int, max_tokens: int, hidden: int, dtype: torch.dtype, device) -> list["FusedAllReduce"]:
        """``world`` ranks' buffers in this process on one GPU; rank r's
        object pushes into all of them. Issue every rank's producer before any
        consumer of the same set (nothing then waits on a later launch)."""
        device = torch.device(device)
        torch.cuda.set_device(device)
        nbytes = cls.buffer_bytes(world, max_tokens, hidden, dtype)
        bufs = [cls._alloc(nbytes) for _ in range(world)]
        objs = [cls(r, world, max_tokens, hidden, dtype, device, bufs[r], bufs, []) for r in range(world)]
        objs[0]._owned = bufs  # rank 0's object frees them all
        for o in objs[1:]:
            o._owned = []
        return objs

    def reset(self) -> None:
        """Re-zero this rank's control words (flags, counters, the broken
        mark) after a timeout; every rank must reset before the next step."""
        _lib.check(_lib.load().ps_comm_reset(self.buf, _lib.stream_ptr(self.device)), "comm_reset")

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib.ps_ipc_close(p)
        for p in self._owned:
            lib.ps_comm_free(p)

    # --------------------------------------------------------- kernels ----
    def linear_push(self, x: torch.Tensor, weight, set_: int, workspace=None, scatter: bool = False) -> None:
        """Row-parallel local product of this rank (x (M, K_shard) @ W.T), pushed
        to every rank's slot ``set_`` (``scatter``: only each rank's column
        slice, to that rank). ``weight``: QuantizedWeight (int8, per-row scale)
        or a bf16/f16 tensor (N, K_shard)."""
        from .quantization import LinearWorkspace, QuantizedWeight, _default_ws
        _lib.require_cuda(x)
        M, K = x.shape
        if M > self.max_tokens:
            raise ValueError(f"{M} tokens exceed the fused all-reduce capacity {self.max_tokens}")
        lib = _lib.load()
        if isinstance(weight, QuantizedWeight):
            N = weight.shape[0]  # int8: the kernels read only the tiled copy
            w_ptr, wdt, wt_ptr, sc_ptr = None, _lib.PS_I8, weight.tiled().data_ptr(), weight.scale.data_ptr()
        else:
            N = weight.shape[0]
            w_ptr, wdt, wt_ptr, sc_ptr = weight.data_ptr(), _lib.dtype_code(weight.dtype), None, None
        if N != self.hidden:
            raise ValueError(f"output width {N} != hidden {self.hidden}")
        ws_bytes = lib.ps_w8a16_linear_tiled_workspace_size(M, N, K)
        if workspace is None:
            workspace = _default_ws.setdefault(x.device, LinearWorkspace())
        buf = workspace.get(ws_bytes, x.device)
        fn = lib.ps_linear_push_scatter if scatter else lib.ps_linear_push
        _lib.check(fn(x.data_ptr(), w_ptr, wdt, wt_ptr, sc_ptr, M, N, K, _lib.dtype_code(x.dtype), self._rank_bufs,
                      self.world, self.rank, set_, self.max_tokens, _lib.ptr(buf), ws_bytes,
                      _lib.stream_ptr(x.device)), "linear_push")

    def linear_push_scatter(self, x: torch.Tensor, weight, set_: int, workspace=None) -> None:
        """Two-shot producer: like :meth:`linear_push`, but each rank receives
        only its own column slice of the output."""
        self.linear_push(x, weight, set_, workspace, scatter=True)

    def gathered_ptr(self, set_: int) -> int:
        """Device address of this rank's gathered residual stream of ``set_``
        ([max_tokens][hidden]; written by ``reduce_norm``)."""
        off = _lib.load().ps_comm_gathered_offset(self.world, self.max_tokens, self.hidden,
                                                  _lib.dtype_code(self.dtype), set_)
        if off == 0:
            raise ValueError("invalid gathered region")
        return self.buf + off

    def gathered(self, set_: int, M: int) -> torch.Tensor:
        """View of the first ``M`` rows of the gathered residual stream of
        ``set_`` (valid until that set's next reduction)."""
        return _lib.device_view(self.gathered_ptr(set_), (M, self.hidden), self.dtype, self.device)

    def reduce_norm(self, x_old: int | torch.Tensor | None, weight: torch.Tensor | None, eps: float, set_: int,
                    M: int, out: torch.Tensor | None = None, phases: int = 3) -> torch.Tensor:
        """Two-shot consumer of ``set_``: the residual stream becomes
        x_old + the reduced sum (left in ``gathered_ptr(set_)``), and the
        return value is rmsnorm(x) * weight for all M rows (x itself when
        ``weight`` is None). ``x_old``: a (M, hidden) tensor, a device
        address with row stride hidden, or None."""
        if out is None:
            out = torch.empty((M, self.hidden), dtype=self.dtype, device=self.device)
        xo = x_old.data_ptr() if isinstance(x_old, torch.Tensor) else x_old
        if weight is not None:
            _lib.require_cuda(weight)
        _lib.check(_lib.load().ps_tp_reduce_rmsnorm(out.data_ptr(), xo, _lib.ptr(weight), float(eps), M, self.hidden,
                                                     _lib.dtype_code(self.dtype), self._rank_bufs, self.world,
                                                     self.rank, set_, self.max_tokens, phases,
                                                     _lib.stream_ptr(self.device)), "tp_reduce_rmsnorm")
        return out

    def allreduce_rmsnorm(self, x: torch.Tensor | None, weight: torch.Tensor | None, eps: float, set_: int,
                          M: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Consume ``set_``: with ``weight``, x += sum of the ranks' slots (in
        place) and return rmsnorm(x) * weight; without, return the sum."""
        H = self.hidden
        if weight is not None:
            _lib.require_cuda(x, weight)
            M = x.shape[0]
        if M is None:
            raise ValueError("M is required without a residual tensor")
        if out is None:
            out = torch.empty((M, H), dtype=self.dtype, device=self.device)
        _lib.check(_lib.load().ps_allreduce_rmsnorm(out.data_ptr(), _lib.ptr(x), _lib.ptr(weight), float(eps), M, H,
                                                     _lib.dtype_code(self.dtype), self.buf, self.world, set_,
                                                     self.max_tokens, _lib.stream_ptr(self.device)),
                   "allreduce_rmsnorm")
        return out

    def row_parallel_linear(self, x_shard: torch.Tensor, weight, set_: int = 0, workspace=None) -> torch.Tensor:
        """engine/tensor_parallel.py:34-48 on this transport: the full (M, N)
        output, identical on every rank. Every rank must call it."""
        self.linear_push(x_shard, weight, set_, workspace)
        return self.allreduce_rmsnorm(None, None, 0.0, set_, M=x_shard.shape[0])
