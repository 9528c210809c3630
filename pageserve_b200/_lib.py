"""ctypes binding of libpageserve_b200.so (the C ABI in include/pageserve_b200.h).

There is no fallback: if the library is missing, or a tensor is not on a CUDA
device, calls raise. Error codes map to the Python exception types the
reference raises for the same condition (IndexError for a short block table,
AssertionError stays with the TP wrappers, ValueError/TypeError for bad
arguments).
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_float, c_int, c_size_t, c_uint64, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libpageserve_b200.so"

PS_F32, PS_BF16, PS_F16, PS_I8 = 0, 1, 2, 3
PS_OK, PS_ERR_INVALID, PS_ERR_INDEX, PS_ERR_CUDA, PS_ERR_UNSUPPORTED, PS_ERR_DEVICE, PS_ERR_TIMEOUT = range(7)

DEVICE_ERRORS = {1: "block id outside the KV pool", 2: "slot outside the cache", 3: "token id outside the vocabulary",
                 4: "bounded device wait timed out", 5: "per-sequence metadata inconsistent with launch bounds"}

_P = c_void_p
_I = c_int
# name -> (restype, argtypes); mirrors include/pageserve_b200.h
_SIGNATURES = {
    "ps_abi_version": (c_int, []),
    "ps_last_error": (ctypes.c_char_p, []),
    "ps_launch_count": (c_uint64, []),
    "ps_device_status": (c_int, [ctypes.POINTER(c_int), _I, _P]),
    "ps_write_kv": (c_int, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "ps_build_slot_mapping": (c_int, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P]),
    "ps_paged_attention_workspace_size": (c_size_t, [_I, _I, _I, _I, _I, _I]),
    "ps_paged_attention": (c_int, [_P, _P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _P,
                                   c_size_t, _P]),
    "ps_paged_attention_noalloc": (c_int, [_P, _P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I,
                                           _P]),
    "ps_quantize_per_channel": (c_int, [_P, _P, _P, _I, _I, _I, _P]),
    "ps_w8a16_linear_workspace_size": (c_size_t, [_I, _I, _I]),
    "ps_w8a16_linear": (c_int, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, c_size_t, _P]),
    "ps_tiled_int8_weight_bytes": (c_size_t, [_I, _I]),
    "ps_tile_int8_weight": (c_int, [_P, _P, _I, _I, _P]),
    "ps_w8a16_linear_tiled_workspace_size": (c_size_t, [_I, _I, _I]),
    "ps_w8a16_linear_tiled": (c_int, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, c_size_t, _P]),
    "ps_linear": (c_int, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, c_size_t, _P]),
    "ps_silu_mul": (c_int, [_P, _P, _I, _I, _I, _P]),
    "ps_rmsnorm": (c_int, [_P, _P, _P, _P, _P, c_float, _I, _I, _I, _P]),
    "ps_apply_rope": (c_int, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "ps_rope_qkv_write_kv": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "ps_embedding": (c_int, [_P, _P, _P, _I, _I, _I, _I, _P]),
    "ps_argmax": (c_int, [_P, _P, _I, _I, _I, _I, _P]),
    "ps_linear_swiglu": (c_int, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _P]),
    "ps_comm_buffer_bytes": (c_size_t, [_I, _I, _I, _I]),
    "ps_comm_alloc": (c_int, [_P, c_size_t]),
    "ps_comm_free": (c_int, [_P]),
    "ps_comm_reset": (c_int, [_P, _P]),
    "ps_ipc_get_handle": (c_int, [_P, _P]),
    "ps_ipc_open_handle": (c_int, [_P, _P]),
    "ps_ipc_close": (c_int, [_P]),
    "ps_linear_push": (c_int, [_P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _P, c_size_t, _P]),
    "ps_allreduce_rmsnorm": (c_int, [_P, _P, _P, c_float, _I, _I, _I, _P, _I, _I, _I, _P]),
    "ps_linear_push_scatter": (c_int, [_P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _P, c_size_t, _P]),
    "ps_tp_reduce_rmsnorm": (c_int, [_P, _P, _P, c_float, _I, _I, _I, _P, _I, _I, _I, _I, _I, _P]),
    "ps_comm_gathered_offset": (c_size_t, [_I, _I, _I, _I, _I]),
    "ps_copy_kv_blocks": (c_int, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P]),
    "ps_topk": (c_int, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "ps_sample_topk": (c_int, [_P, _P, _P, _P, _I, _I, c_float, _P]),
}

_lock = threading.Lock()
_lib = None
_status_ready: set[int] = set()


def load() -> ctypes.CDLL:
    """Load the library once (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("PAGESERVE_B200_LIB", LIB_PATH))
            if not path.exists():
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m pageserve_b200.build` "
                    "(pageserve_b200 has no CPU fallback)")
            lib = ctypes.CDLL(str(path))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class _DeviceArray:
    """__cuda_array_interface__ over raw device memory this library owns."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3}


def device_view(ptr: int, shape: tuple, dtype, device) -> "object":
    """A torch tensor viewing device memory at ``ptr`` (no copy; the memory
    must outlive the view). 16-bit dtypes are viewed through int16."""
    import torch
    n = 1
    for d in shape:
        n *= d
    raw = torch.as_tensor(_DeviceArray(ptr, (n,), "<i2"), device=device)
    return raw.view(dtype).view(*shape)


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    return load().ps_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == PS_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == PS_ERR_INDEX:
        raise IndexError(msg)
    if rc == PS_ERR_INVALID:
        raise ValueError(msg)
    if rc == PS_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == PS_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return PS_BF16
    if dt == torch.float16:
        return PS_F16
    if dt == torch.float32:
        return PS_F32
    if dt == torch.int8:
        return PS_I8
    raise TypeError(f"pageserve_b200: unsupported dtype {dt}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("pageserve_b200 kernels run on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ensure_status_word(device: torch.device) -> None:
    """Allocate the device status word outside any graph capture."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx in _status_ready:
        return
    with torch.cuda.device(idx):
        code = c_int(0)
        check(load().ps_device_status(ctypes.byref(code), 1, None), "device_status")
    _status_ready.add(idx)


def device_status(clear: bool = True) -> int:
    """Synchronise the current stream and return the device status code."""
    code = c_int(0)
    check(load().ps_device_status(ctypes.byref(code), 1 if clear else 0, stream_ptr()), "device_status")
    return code.value


def raise_on_device_error() -> None:
    code = device_status(clear=True)
    if code:
        raise RuntimeError(f"pageserve_b200 device error {code}: {DEVICE_ERRORS.get(code, 'unknown')}")


def launch_count() -> int:
    return int(load().ps_launch_count())
