"""Helpers for the GPU parity tests: device buffers via torch (plumbing only)
and direct calls into libtfx's C ABI."""

from __future__ import annotations

import ctypes

import numpy as np
import torch

import tfx
from tfx import _lib


def dev(a: np.ndarray, offset_elems: int = 0) -> torch.Tensor:
    """Upload a numpy array; offset_elems > 0 places it off the 16-byte grid."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if offset_elems:
        buf = torch.empty(t.numel() + offset_elems, dtype=t.dtype, device="cuda")
        view = buf[offset_elems:]
        view.copy_(t.reshape(-1))
        return view
    return t.cuda()


def empty(n: int, dtype=torch.float32, offset_elems: int = 0) -> torch.Tensor:
    if offset_elems:
        return torch.empty(n + offset_elems, dtype=dtype, device="cuda")[offset_elems:]
    return torch.empty(n, dtype=dtype, device="cuda")


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def S():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def call(name: str, *args) -> None:
    rc = getattr(_lib.lib, name)(*args)
    if rc != 0:
        raise tfx.TfxError(rc, tfx.last_error())


def f32(v):
    return ctypes.c_float(v)


def f64(v):
    return ctypes.c_double(v)
