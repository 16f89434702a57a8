"""Tensor checks, stream handles and per-stream workspaces for the libftb calls."""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_WS: dict = {}


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise ValueError(f"ftb ops run on CUDA tensors only (got {dev}); there is no CPU path")
    for t in tensors:
        if t.device != dev:
            raise ValueError(f"all tensors must be on {dev} (got {t.device})")
    return dev


def require(t: torch.Tensor, name: str, dtype=None, shape=None, contiguous=True) -> None:
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A cached uint8 device buffer of at least ``nbytes`` for the current stream.

    Grown (never shrunk) on demand; call once eagerly before CUDA-graph capture so capture
    does not allocate. Calls on one stream are ordered, so sharing it per stream is safe."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    t = _WS.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(int(nbytes), 1 << 16), dtype=torch.uint8, device=device)
        _WS[key] = t
    return t


def read_status(ws: torch.Tensor) -> int:
    """The device status word (first 4 bytes of a workspace); synchronises the stream."""
    return int(ws[:4].view(torch.int32).item())


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())
