"""Host-side helpers shared by the API modules: dtype codes, the caller's stream,
per-device cached buffers (workspaces, constant length vectors)."""

from __future__ import annotations

import torch

from . import _lib

_DTYPE_CODES = {torch.float32: _lib.SPA_F32, torch.float16: _lib.SPA_F16, torch.bfloat16: _lib.SPA_BF16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from None


def stream_ptr(device: torch.device | int) -> int:
    """The raw handle of the caller's current stream on ``device`` (a device or its index)."""
    index = device if isinstance(device, int) else device.index
    if index is None:
        index = torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(index)


def require_cuda(*tensors: torch.Tensor, message: str = "CUDA tensors are required") -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(message)


def require_contiguous(*tensors: torch.Tensor, message: str = "contiguous CUDA tensors are required") -> None:
    for t in tensors:
        if t is not None and not t.is_contiguous():
            raise ValueError(message)


_WORKSPACES: dict[tuple, torch.Tensor] = {}
_CONST_I32: dict[tuple, torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A device byte buffer of at least ``nbytes`` reserved for the caller's current
    stream (one buffer per (device, stream); calls on one stream are ordered, so the
    buffer is never used by two kernels at once).  The decode kernels write every
    partial they read back, so no initial contents are needed."""
    key = (device.index, stream_ptr(device))
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf


def const_i32(device: torch.device, n: int, value: int) -> torch.Tensor:
    """A cached int32 device vector of length n filled with value (read-only use)."""
    key = (device.index, n, value)
    t = _CONST_I32.get(key)
    if t is None:
        t = torch.full((n,), value, dtype=torch.int32, device=device)
        _CONST_I32[key] = t
    return t


def as_int64(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.int64:
        return t
    if t.dtype == torch.int32:
        return t.to(torch.int64)
    raise ValueError(f"page indices must be int32 or int64, got {t.dtype}")


def as_int32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.int32:
        return t
    if t.dtype == torch.int64:
        return t.to(torch.int32)
    raise ValueError(f"page table / lengths must be int32 or int64, got {t.dtype}")
