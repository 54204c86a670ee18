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


FRESH_SCHEMA = (
    "take_top_k_and_gather_from_main_and_fresh(Tensor main_scores, Tensor fresh_scores, Tensor main_indices, "
    "Tensor fresh_indices, int k, str[] keys, Tensor[] list_main_data, Tensor[] list_fresh_data, "
    "int kernel_version=2) -> (Tensor, Tensor, Tensor, Dict(str, Tensor))"
)


def take_top_k_and_gather_from_main_and_fresh(main_scores: Tensor, fresh_scores: Tensor, main_indices: Tensor,
                                              fresh_indices: Tensor, k: int, keys: list[str],
                                              list_main_data: list[Tensor], list_fresh_data: list[Tensor],
                                              kernel_version: int = 2):
    """``st::take_top_k_and_gather_from_main_and_fresh`` (fresh_index_post_processing.cpp:226-272):
    ``(top_scores [B, k'], top columns int64 [B, k'] into [fresh | main], is_from_fresh bool,
    {key: the winners' data rows [B k', ...]})``, ``k' = min(k, Mf + Mm)``; largest first, NaN the
    largest, ties to the lower merged column (torch.topk, which the reference calls, leaves tie
    order open). ``kernel_version`` picks a kernel upstream and changes nothing here."""
    _check(len(keys) == len(list_main_data),
           f"keys and list_main_data should have the same size. keys.size()={len(keys)}, "
           f"list_main_data.size()={len(list_main_data)}")
    _check(len(keys) == len(list_fresh_data),
           f"keys and list_fresh_data should have the same size. keys.size()={len(keys)}, "
           f"list_fresh_data.size()={len(list_fresh_data)}")
    for key, md, fd in zip(keys, list_main_data, list_fresh_data):
        _check(md.dim() == fd.dim(), f"main_data and fresh_data should have the same dim. key={key}")
        _check(0 < md.dim() <= 2, f"The main data dim must be in [1, 2], main_data.dim()={md.dim()}")
        if md.dim() > 1:
            _check(md.shape[-1] == fd.shape[-1],
                   f"main_data and fresh_data should have the same number of element in the last dim. key={key}")
        _check(md.dtype == fd.dtype, f"main_data and fresh_data should have the same scalar_type. key={key}")
        _check(md.is_cuda and fd.is_cuda, f"the data of key {key} must be CUDA tensors")
    for name, t in (("main_scores", main_scores), ("fresh_scores", fresh_scores), ("main_indices", main_indices),
                    ("fresh_indices", fresh_indices)):
        _check(t.is_cuda and t.dim() == 2, f"{name} must be a 2-D CUDA tensor")
    _check(main_scores.dtype == fresh_scores.dtype and main_scores.dtype in _DTYPES,
           "main_scores and fresh_scores must share a float dtype")
    _check(main_indices.shape == main_scores.shape and fresh_indices.shape == fresh_scores.shape,
           "each indices tensor must have its scores' shape")
    _check(main_indices.dtype == fresh_indices.dtype and main_indices.dtype in (torch.int32, torch.int64),
           "main_indices and fresh_indices must share an int32 or int64 dtype")
    b, mm = main_scores.shape
    mf = fresh_scores.shape[1]
    _check(fresh_scores.shape[0] == b, "main and fresh scores must have the same rows")
    dev = main_scores.device
    kk = max(0, min(int(k), mf + mm))
    top_scores = torch.empty((b, kk), dtype=main_scores.dtype, device=dev)
    top_idx = torch.empty((b, kk), dtype=torch.int64, device=dev)
    is_fresh = torch.empty((b, kk), dtype=torch.bool, device=dev)
    lib = _lib.lib()
    what = "st::take_top_k_and_gather_from_main_and_fresh"
    ms, fs = main_scores.contiguous(), fresh_scores.contiguous()
    _call(lib.rb_st_fresh_topk(_ptr(fs), mf, _ptr(ms), mm, _DTYPES[ms.dtype], b, kk, _ptr(top_scores), _ptr(top_idx),
                               _ptr(is_fresh), _stream(dev)), what)
    mi, fi = main_indices.contiguous(), fresh_indices.contiguous()
    gathered = {}
    for key, md, fd in zip(keys, list_main_data, list_fresh_data):
        md, fd = md.contiguous(), fd.contiguous()
        row_elems = md.shape[1] if md.dim() == 2 else 1
        shape = (b * kk, row_elems) if md.dim() == 2 else (b * kk,)
        out = torch.zeros(shape, dtype=md.dtype, device=dev)
        _call(lib.rb_st_fresh_gather(_ptr(top_idx), b, kk, mf, mm, _ptr(fi), _ptr(mi), int(mi.dtype == torch.int64),
                                     _ptr(fd), fd.shape[0], _ptr(md), md.shape[0], row_elems, md.element_size(),
                                     _ptr(out), _stream(dev)), what)
        gathered[key] = out
    return top_scores, top_idx, is_fresh, gathered


def _fake_fresh(main_scores, fresh_scores, main_indices, fresh_indices, k, keys, list_main_data, list_fresh_data,
                kernel_version=2):
    b = main_scores.shape[0]
    kk = max(0, min(int(k), main_scores.shape[1] + fresh_scores.shape[1]))
    data = {key: md.new_empty((b * kk, md.shape[1]) if md.dim() == 2 else (b * kk,))
            for key, md in zip(keys, list_main_data)}
    return (main_scores.new_empty((b, kk)), main_scores.new_empty((b, kk), dtype=torch.int64),
            main_scores.new_empty((b, kk), dtype=torch.bool), data)


OPS = (("is_topk", IS_TOPK_SCHEMA, is_topk, _fake_is_topk),
       ("take_top_k_and_gather_from_main_and_fresh", FRESH_SCHEMA, take_top_k_and_gather_from_main_and_fresh,
        _fake_fresh))
