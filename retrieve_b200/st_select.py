"""``torch.ops.st.is_topk`` on ``libretrieve_b200.so``: the top-k membership flags of
SilverTorch's extension (silvertorch/ops/csrc/is_topk.cpp:84-90, CUDA is_topk_cuda.cu:83-149),
with the CUDA op's semantics: per row the value at sorted position ``clamp(k - 1, 0, n - 1)``
(descending, or ascending with ``largest=False``; NaN sorts as the largest value) and every score
at or beyond it flagged 1 in ``is_topk_output`` (the scores' dtype), compared in fp32. Ties at the
k-th value are all flagged. Errors raise ``RuntimeError``."""

from __future__ import annotations

import torch
from torch import Tensor

from retrieve_b200 import _lib
from retrieve_b200._st_common import _call, _check, _ptr, _stream

IS_TOPK_SCHEMA = "is_topk(Tensor scores, Tensor ks, Tensor(a!) is_topk_output, bool largest=True) -> ()"

_DTYPES = {torch.float32: _lib.RB_F32, torch.float16: _lib.RB_F16, torch.bfloat16: _lib.RB_BF16}


def is_topk(scores: Tensor, ks: Tensor, is_topk_output: Tensor, largest: bool = True) -> None:
    # the reference's checks, is_topk_cuda.cu:89-101
    _check(scores.is_cuda, "scores must be on CUDA")
    _check(ks.is_cuda, "ks must be on CUDA")
    _check(is_topk_output.is_cuda, "is_topk_output must be on CUDA")
    _check(scores.dim() == 2, "scores must be 2D tensor")
    _check(ks.dim() == 1, "ks must be 1D tensor")
    _check(ks.shape[0] == scores.shape[0], "ks size must match scores batch size")
    _check(is_topk_output.is_contiguous(), "is_topk_output must be contiguous")
    _check(tuple(is_topk_output.shape) == tuple(scores.shape), "is_topk_output must have same shape as scores")
    _check(scores.dtype in _DTYPES, f"unsupported score dtype {scores.dtype}")
    _check(is_topk_output.dtype == scores.dtype, "is_topk_output must have the scores' dtype")
    s = scores.contiguous()
    k = ks.to(torch.int64).contiguous()
    b, n = s.shape
    _call(_lib.lib().rb_st_is_topk(_ptr(s), _DTYPES[s.dtype], b, n, _ptr(k), int(bool(largest)),
                                   _ptr(is_topk_output), _stream(s.device)), "st::is_topk")


def _fake_is_topk(scores, ks, is_topk_output, largest=True):
    return None


OPS = (("is_topk", IS_TOPK_SCHEMA, is_topk, _fake_is_topk),)
