"""``st::is_topk`` (retrieve_b200/st_select.py, csrc/is_topk.cu) against its restatement
(oracle/select.py), which follows the reference's CUDA op: the k-th value from a sort with NaN as
the largest, every score at or beyond it flagged, ties included, k clamped to [1, n]."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import select

PINNED = "st::is_topk(Tensor scores, Tensor ks, Tensor(a!) is_topk_output, bool largest=True) -> ()"


def _st():
    import retrieve_b200.st  # noqa: F401  (registers the ops)

    return torch.ops.st


def test_schema_is_the_reference_one():
    # silvertorch/ops/csrc/is_topk.cpp:84-90
    assert str(_st().is_topk.default._schema) == PINNED


def test_restatement_follows_the_cuda_op():
    """Ties at the k-th value are all flagged; k <= 0 takes the largest value (the CUDA op clamps
    k - 1 to 0, where the CPU op flags nothing) and k >= n every finite score; a NaN k-th value
    flags nothing."""
    s = np.array([[3, 1, 3, 2, 0], [5, 4, 3, 2, 1], [1, 2, np.nan, 0, 2], [1, 2, 3, 4, 5]], dtype=np.float32)
    out = select.is_topk(s, [2, 0, 1, 9])
    assert out.tolist() == [[1, 0, 1, 0, 0], [1, 0, 0, 0, 0], [0, 0, 0, 0, 0], [1, 1, 1, 1, 1]]
    low = select.is_topk(s, [2, 1, 2, 2], largest=False)
    assert low.tolist() == [[0, 1, 0, 0, 1], [0, 0, 0, 0, 1], [1, 0, 0, 1, 0], [1, 1, 0, 0, 0]]


def test_cpu_tensors_raise():
    _st()
    from retrieve_b200 import st_select

    s = torch.zeros(2, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        st_select.is_topk(s, torch.ones(2, dtype=torch.int64), torch.zeros(2, 3))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("largest", [True, False])
def test_is_topk_matches_restatement(dtype, largest):
    st = _st()
    g = torch.Generator().manual_seed(3)
    s = torch.randn(40, 3000, generator=g)
    s[:, :500] = torch.round(s[:, :500] * 2) / 2  # many ties
    s[3, 7] = float("nan")
    s[5] = float("nan")
    s[6, :10] = float("-inf")
    s = s.to(dtype)
    ks = torch.randint(-2, 3200, (40,), generator=g)
    ks[0], ks[1] = 1, 3000
    out = torch.full(s.shape, 7.0, dtype=dtype, device="cuda")
    st.is_topk(s.cuda(), ks.cuda(), out, largest)
    want = select.is_topk(s.float().numpy(), ks.numpy(), largest)
    assert np.array_equal(out.float().cpu().numpy(), want)
