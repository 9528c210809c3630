"""Drop-in for the reference's engine/quantization.py with a fused W8A16 kernel.

``QuantizedWeight`` keeps the reference's attributes (``q`` int8 (N, K),
``scale`` float32 (N, 1), ``dtype``, ``get()``, ``to()``, ``storage_bytes``)
so loaders and tests are unchanged, and adds ``linear(x, bias, residual)``:
y = x @ (q * scale).T + bias (+ residual) computed by the sm_100a kernel
without ever materialising the dequantized weight (the reference
re-dequantizes the whole weight on every ``get()``,
engine/quantization.py:40-41).
"""

from __future__ import annotations

import torch

from . import _lib


def _cuda_device(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("pageserve_b200 quantizes on the GPU (no CPU fallback); no CUDA device is available")
    return torch.device("cuda", torch.cuda.current_device())


def quantize_per_channel(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """engine/quantization.py:16-23, bit-exact, computed on the GPU:
    scale = max(absmax_k, 1e-8) / 127 (float32, (N, 1)),
    q = clamp(round_half_even(w / scale), -127, 127) int8 (N, K).
    Results live on the weight's CUDA device (a CPU weight is moved to the
    current CUDA device first)."""
    dev = _cuda_device(weight)
    w = weight.to(dev).contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        w = w.float()
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.int8, device=dev)
    scale = torch.empty((N, 1), dtype=torch.float32, device=dev)
    _lib.check(_lib.load().ps_quantize_per_channel(q.data_ptr(), scale.data_ptr(), w.data_ptr(),
                                                   _lib.dtype_code(w.dtype), N, K, _lib.stream_ptr(dev)),
               "quantize_per_channel")
    return q, scale


def dequantize(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """engine/quantization.py:26-27 (materialises the weight; the fused
    kernel path never calls this)."""
    return (q.to(torch.float32) * scale).to(dtype)


class LinearWorkspace:
    """Grow-only scratch buffer of the tensor-core linear: the float32
    partial tiles that the split-K CTAs of an output tile exchange through L2
    (each call writes every slot it reads, so no clearing is needed). One
    buffer serves all the linears of a step (calls on one stream only);
    without it the splits reduce through shared memory, more slowly."""

    def __init__(self):
        self.buf: torch.Tensor | None = None

    def get(self, nbytes: int, device) -> torch.Tensor | None:
        if nbytes == 0:
            return None
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != torch.device(device):
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        return self.buf


_default_ws: dict[torch.device, LinearWorkspace] = {}


def tile_int8_weight(q: torch.Tensor) -> torch.Tensor:
    """Kernel-side copy of an int8 weight [N][K] in contiguous 8 KB blocks
    [ceil(N/128)][ceil(K/64)][128][64] (zero padded), streamed by the
    tensor-core linear with one bulk copy per block."""
    _lib.require_cuda(q)
    N, K = q.shape
    lib = _lib.load()
    out = torch.empty(lib.ps_tiled_int8_weight_bytes(N, K), dtype=torch.int8, device=q.device)
    _lib.check(lib.ps_tile_int8_weight(out.data_ptr(), q.contiguous().data_ptr(), N, K, _lib.stream_ptr(q.device)),
               "tile_int8_weight")
    return out


def untile_int8_weight(tiled: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """Inverse of :func:`tile_int8_weight`: the row-major [N][K] int8 weight
    from the 8 KB-block layout, where 16-byte chunk c of row r of a block is
    stored at chunk slot c ^ ((r >> 1) & 3). Plain tensor indexing (any
    device); the model keeps only the tiled copy and rebuilds the row-major
    one when a caller asks for ``QuantizedWeight.q``."""
    nb, kt = (N + 127) // 128, (K + 63) // 64
    t = tiled.view(nb, kt, 128, 4, 16)
    r = torch.arange(128, device=tiled.device).view(128, 1)
    c = torch.arange(4, device=tiled.device).view(1, 4)
    blocks = t[:, :, r, c ^ ((r >> 1) & 3)]  # [nb][kt][128][4][16], chunks back in order
    return blocks.permute(0, 2, 1, 3, 4).reshape(nb * 128, kt * 64)[:N, :K].contiguous()


def w8a16_linear(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None,
                 residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 workspace: LinearWorkspace | None = None, q_tiled: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ (q * scale).T + bias (+ residual): F.linear(x, QuantizedWeight.get(), bias)
    of engine/model.py:168-190, fused. x (..., K) bf16/f16/f32 on CUDA.
    With ``q_tiled`` (from :func:`tile_int8_weight`) and a 16-bit x, the
    tensor-core kernel streams the pre-tiled copy."""
    _lib.require_cuda(x, q, scale, bias, residual)
    N, K = q.shape
    if q_tiled is not None and x.dtype in (torch.bfloat16, torch.float16):
        return _w8a16_tiled(x, q_tiled, scale, N, K, bias, residual, out, workspace)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    if residual is not None:
        residual = residual.reshape(M, N).contiguous()
    if bias is not None:
        bias = bias.to(x.dtype).contiguous()
    lib = _lib.load()
    ws_bytes = lib.ps_w8a16_linear_workspace_size(M, N, K)
    if workspace is None:
        workspace = _default_ws.setdefault(x.device, LinearWorkspace())
    buf = workspace.get(ws_bytes, x.device)
    _lib.check(lib.ps_w8a16_linear(out.data_ptr(), x2.data_ptr(), q.data_ptr(), scale.data_ptr(), _lib.ptr(bias),
                                   _lib.ptr(residual), M, N, K, _lib.dtype_code(x.dtype), _lib.ptr(buf), ws_bytes,
                                   _lib.stream_ptr(x.device)), "w8a16_linear")
    return out


def _w8a16_tiled(x, q_tiled, scale, N, K, bias, residual, out, workspace):
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    if residual is not None:
        residual = residual.reshape(M, N).contiguous()
    if bias is not None:
        bias = bias.to(x.dtype).contiguous()
    lib = _lib.load()
    ws_bytes = lib.ps_w8a16_linear_tiled_workspace_size(M, N, K)
    if workspace is None:
        workspace = _default_ws.setdefault(x.device, LinearWorkspace())
    buf = workspace.get(ws_bytes, x.device)
    _lib.check(lib.ps_w8a16_linear_tiled(out.data_ptr(), x2.data_ptr(), q_tiled.data_ptr(), scale.data_ptr(),
                                         _lib.ptr(bias), _lib.ptr(residual), M, N, K, _lib.dtype_code(x.dtype),
                                         _lib.ptr(buf), ws_bytes, _lib.stream_ptr(x.device)), "w8a16_linear_tiled")
    return out


def linear16(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
             residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
             workspace: LinearWorkspace | None = None) -> torch.Tensor:
    """F.linear(x, w, bias) with a bf16/f16 weight (the unquantized lm_head,
    engine/model.py:193)."""
    _lib.require_cuda(x, w, bias, residual)
    N, K = w.shape
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    if residual is not None:
        residual = residual.reshape(M, N).contiguous()
    lib = _lib.load()
    ws_bytes = lib.ps_w8a16_linear_workspace_size(M, N, K)
    if workspace is None:
        workspace = _default_ws.setdefault(x.device, LinearWorkspace())
    buf = workspace.get(ws_bytes, x.device)
    _lib.check(lib.ps_linear(out.data_ptr(), x2.data_ptr(), w.data_ptr(), _lib.ptr(bias), _lib.ptr(residual), M, N,
                             K, _lib.dtype_code(x.dtype), _lib.ptr(buf), ws_bytes, _lib.stream_ptr(x.device)),
               "linear")
    return out


def linear_swiglu(x: torch.Tensor, weight, out: torch.Tensor | None = None) -> torch.Tensor:
    """F.silu(F.linear(x, gate_w)) * F.linear(x, up_w) (engine/model.py:188-190)
    in one tensor-core linear over the row-interleaved gate|up weight
    (row 2i = gate row i, row 2i+1 = up row i): ``weight`` is a
    QuantizedWeight of that [2I][K] matrix or a bf16/f16 tensor. Returns
    (..., I)."""
    _lib.require_cuda(x)
    lib = _lib.load()
    if isinstance(weight, QuantizedWeight):
        N2, K = weight.shape  # int8: the kernels read only the tiled copy
        w_ptr, wdt, wt_ptr, sc_ptr = None, _lib.PS_I8, weight.tiled().data_ptr(), weight.scale.data_ptr()
    else:
        N2, K = weight.shape
        w_ptr, wdt, wt_ptr, sc_ptr = weight.data_ptr(), _lib.dtype_code(weight.dtype), None, None
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty((*lead, N2 // 2), dtype=x.dtype, device=x.device)
    _lib.check(lib.ps_linear_swiglu(out.data_ptr(), x2.data_ptr(), w_ptr, wdt, wt_ptr, sc_ptr, M, N2, K,
                                    _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device)), "linear_swiglu")
    return out


class QuantizedWeight:
    """engine/quantization.py:30-50, same attributes; ``linear`` runs the
    fused W8A16 kernel.

    Storage: the row-major int8 ``q`` and/or the kernels' tiled copy
    (:meth:`tiled`). :meth:`release_row_major` keeps only the tiled copy
    (one int8 copy of the weight in HBM); ``q`` is then rebuilt from it on
    each access (exact, for callers outside the hot path)."""

    _q = None
    _tiled = None
    _shape = (0, 0)

    def __init__(self, weight: torch.Tensor):
        self.dtype = weight.dtype
        self.q, self.scale = quantize_per_channel(weight)

    @classmethod
    def from_quantized(cls, q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> "QuantizedWeight":
        obj = cls.__new__(cls)
        obj.dtype = dtype
        obj.q = q.contiguous()
        obj.scale = scale.reshape(-1, 1).to(torch.float32).contiguous()
        return obj

    @property
    def q(self) -> torch.Tensor:
        if self._q is not None:
            return self._q
        return untile_int8_weight(self._tiled, *self._shape)

    @q.setter
    def q(self, value: torch.Tensor) -> None:
        self._q = value
        self._shape = tuple(value.shape)
        self._tiled = None

    def release_row_major(self) -> None:
        """Keep only the tiled copy (built first if needed)."""
        self.tiled()
        self._q = None

    def get(self) -> torch.Tensor:
        return dequantize(self.q, self.scale, self.dtype)

    def to(self, device) -> "QuantizedWeight":
        if self._q is not None:
            self.q = self._q.to(device)
        else:
            self._tiled = self._tiled.to(device)
        self.scale = self.scale.to(device)
        return self

    @property
    def storage_bytes(self) -> int:
        """Bytes of the int8 weight and its scales (the reference's count)."""
        n, k = self._shape
        return n * k + self.scale.numel() * self.scale.element_size()

    @property
    def shape(self) -> tuple[int, int]:
        return tuple(self._shape)

    def tiled(self) -> torch.Tensor:
        """The kernel-side 8 KB-block copy of ``q`` (built once, cached)."""
        t = self._tiled
        if t is None or (self._q is not None and t.device != self._q.device):
            t = tile_int8_weight(self._q)
            self._tiled = t
        return t

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None, workspace: LinearWorkspace | None = None) -> torch.Tensor:
        if x.dtype in (torch.bfloat16, torch.float16):
            _lib.require_cuda(x, self.scale, bias, residual)
            return _w8a16_tiled(x, self.tiled(), self.scale, *self._shape, bias, residual, out, workspace)
        return w8a16_linear(x, self.q, self.scale, bias, residual, out, workspace)


class RowView(QuantizedWeight):
    """Rows ``rows`` (a slice, step 1 or 2) of another QuantizedWeight: the
    reference-facing per-projection weights of a model whose fused q|k|v and
    gate|up weights hold the data. ``q`` and ``get()`` read through to the
    source; :meth:`tiled` is a view of the source's tiled copy when the rows
    are whole 128-row blocks, else a tiled copy of its own."""

    def __init__(self, src: QuantizedWeight, rows: slice, dtype: torch.dtype):
        self.dtype = dtype
        self._src = src
        self._rows = rows
        self.scale = src.scale[rows].contiguous()
        self._shape = (len(range(*rows.indices(src.shape[0]))), src.shape[1])

    @property
    def q(self) -> torch.Tensor:
        """The view's rows, row-major (rebuilt on each access, outside the hot
        path): a step-1 view untiles only the 128-row blocks it covers."""
        if self._q is not None:
            return self._q
        start, stop, step = self._rows.indices(self._src.shape[0])
        src_tiled = self._src._tiled
        if step == 1 and self._src._q is None and src_tiled is not None:
            N, K = self._src.shape
            b0, b1 = start // 128, (stop + 127) // 128
            blk = ((K + 63) // 64) * 8192
            rows = untile_int8_weight(src_tiled[b0 * blk:b1 * blk], (b1 - b0) * 128, K)
            return rows[start - b0 * 128:stop - b0 * 128].contiguous()
        return self._src.q[self._rows].contiguous()

    @q.setter
    def q(self, value: torch.Tensor) -> None:  # an explicit assignment detaches the view
        self._q = value
        self._shape = tuple(value.shape)
        self._tiled = None

    def tiled(self) -> torch.Tensor:
        """A view of the source's tiled copy when the rows are whole 128-row
        blocks; otherwise a temporary tiled copy, rebuilt on every call and
        never cached, so the model keeps one int8 copy of each weight (such
        views, e.g. the step-2 gate/up rows, are slow paths for callers
        outside the hot path)."""
        if self._q is None:
            start, stop, step = self._rows.indices(self._src.shape[0])
            N, K = self._src.shape
            if step == 1 and start % 128 == 0 and (stop % 128 == 0 or stop == N):
                blk = ((K + 63) // 64) * 8192
                return self._src.tiled()[(start // 128) * blk:((stop + 127) // 128) * blk]
            return tile_int8_weight(self.q)
        if self._tiled is None:
            self._tiled = tile_int8_weight(self._q)
        return self._tiled

    def to(self, device) -> "QuantizedWeight":
        return QuantizedWeight.from_quantized(self.q.to(device), self.scale.to(device), self.dtype)
