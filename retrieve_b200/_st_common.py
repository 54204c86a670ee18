"""Argument plumbing shared by the ``torch.ops.st`` implementations: raw pointers, the
caller's stream, and the reference's error convention (``TORCH_CHECK`` raises
``RuntimeError``; a non-zero C-ABI status becomes one with the library's message)."""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from retrieve_b200 import _lib


def _ptr(t: Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _call(rc: int, what: str) -> None:
    if rc != _lib.RB_OK:
        msg = _lib.lib().rb_last_error().decode(errors="replace")
        raise RuntimeError(f"{what}: {msg} (status {rc})")


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)
