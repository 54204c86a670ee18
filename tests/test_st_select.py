"""SilverTorch's selection ops ``st::is_topk`` and ``st::take_top_k_and_gather_from_main_and_fresh``
(retrieve_b200/st_select.py, csrc/is_topk.cu, csrc/fresh_merge.cu) against their restatements
(oracle/select.py), which follow the reference's CUDA ops and are pinned to its CPU ops
(tests/golden/golden_select.npz, made by tests/golden/make_golden_select.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import select

PINNED = "st::is_topk(Tensor scores, Tensor ks, Tensor(a!) is_topk_output, bool largest=True) -> ()"
PINNED_FRESH = (  # fresh_index_post_processing.cpp:275-286
    "st::take_top_k_and_gather_from_main_and_fresh(Tensor main_scores, Tensor fresh_scores, "
    "Tensor main_indices, Tensor fresh_indices, int k, str[] keys, Tensor[] list_main_data, "
    "Tensor[] list_fresh_data, int kernel_version=2) -> (Tensor, Tensor, Tensor, Dict(str, Tensor))"
)
GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden_select.npz")


def _st():
    import retrieve_b200.st  # noqa: F401  (registers the ops)

    return torch.ops.st


def test_schema_is_the_reference_one():
    # silvertorch/ops/csrc/is_topk.cpp:84-90
    assert str(_st().is_topk.default._schema) == PINNED
    assert str(_st().take_top_k_and_gather_from_main_and_fresh.default._schema) == PINNED_FRESH


@pytest.mark.parametrize("largest", [True, False])
def test_is_topk_restatement_matches_reference(largest):
    got = select.is_topk(GOLDEN["is_topk_scores"], GOLDEN["is_topk_ks"], largest)
    assert np.array_equal(got, GOLDEN[f"is_topk_{int(largest)}"])


def _fresh_args():
    g = GOLDEN
    return g["main_scores"], g["fresh_scores"], g["main_idx"], g["fresh_idx"]


@pytest.mark.parametrize("k", [7, 60])
def test_take_top_k_restatement_matches_reference(k):
    for key, md, fd in (("emb", GOLDEN["main_emb"], GOLDEN["fresh_emb"]), ("id", GOLDEN["main_id"], GOLDEN["fresh_id"])):
        top, cols, fresh, data = select.take_top_k_and_gather(*_fresh_args(), k, md, fd)
        assert np.array_equal(top.astype(np.float32), GOLDEN[f"ttk{k}_top"])
        assert np.array_equal(cols, GOLDEN[f"ttk{k}_cols"]) and np.array_equal(fresh, GOLDEN[f"ttk{k}_fresh"])
        assert np.array_equal(data, GOLDEN[f"ttk{k}_{key}"])


def test_take_top_k_argument_errors_and_fakes():
    st = _st()
    from torch._subclasses.fake_tensor import FakeTensorMode

    from retrieve_b200 import st_select

    z = torch.zeros(2, 3)
    i = torch.zeros(2, 3, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="same size"):
        st_select.take_top_k_and_gather_from_main_and_fresh(z, z, i, i, 2, ["a"], [], [])
    with pytest.raises(RuntimeError, match="same dim"):
        st_select.take_top_k_and_gather_from_main_and_fresh(z, z, i, i, 2, ["a"], [torch.zeros(4)],
                                                            [torch.zeros(4, 2)])
    with FakeTensorMode():
        top, cols, fresh, data = st.take_top_k_and_gather_from_main_and_fresh(
            torch.empty(2, 30), torch.empty(2, 5), torch.empty(2, 30, dtype=torch.int64),
            torch.empty(2, 5, dtype=torch.int64), 50, ["e", "i"], [torch.empty(9, 4), torch.empty(9)],
            [torch.empty(3, 4), torch.empty(3)])
        assert top.shape == cols.shape == fresh.shape == (2, 35) and fresh.dtype == torch.bool
        assert data["e"].shape == (70, 4) and data["i"].shape == (70,)


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


@pytest.mark.gpu
@pytest.mark.parametrize("largest", [True, False])
def test_is_topk_matches_reference_fixture(largest):
    st = _st()
    s = torch.from_numpy(GOLDEN["is_topk_scores"]).cuda()
    out = torch.zeros_like(s)
    st.is_topk(s, torch.from_numpy(GOLDEN["is_topk_ks"]).cuda(), out, largest)
    assert np.array_equal(out.cpu().numpy(), GOLDEN[f"is_topk_{int(largest)}"])


@pytest.mark.gpu
@pytest.mark.parametrize("k", [7, 60])
def test_take_top_k_matches_reference_fixture(k):
    st = _st()
    dev = [torch.from_numpy(a).cuda() for a in _fresh_args()]
    top, cols, fresh, data = st.take_top_k_and_gather_from_main_and_fresh(
        *dev, k, ["emb", "id"], [torch.from_numpy(GOLDEN["main_emb"]).cuda(), torch.from_numpy(GOLDEN["main_id"]).cuda()],
        [torch.from_numpy(GOLDEN["fresh_emb"]).cuda(), torch.from_numpy(GOLDEN["fresh_id"]).cuda()])
    assert np.array_equal(top.cpu().numpy(), GOLDEN[f"ttk{k}_top"])
    assert np.array_equal(cols.cpu().numpy(), GOLDEN[f"ttk{k}_cols"])
    assert np.array_equal(fresh.cpu().numpy(), GOLDEN[f"ttk{k}_fresh"])
    assert np.array_equal(data["emb"].cpu().numpy(), GOLDEN[f"ttk{k}_emb"])
    assert np.array_equal(data["id"].cpu().numpy(), GOLDEN[f"ttk{k}_id"])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_take_top_k_ties_and_nan(dtype):
    """Tied scores go to the lower merged column (fresh first), NaN ranks first; int32 indices."""
    st = _st()
    g = torch.Generator().manual_seed(2)
    main = torch.round(torch.randn(16, 700, generator=g) * 2) / 2
    fresh = torch.round(torch.randn(16, 90, generator=g) * 2) / 2
    main[3, 5] = float("nan")
    fresh[4, 0] = float("nan")
    mi = torch.randint(-5, 500, (16, 700), generator=g, dtype=torch.int32)
    fi = torch.randint(-5, 50, (16, 90), generator=g, dtype=torch.int32)
    md, fd = torch.randn(500, 3, generator=g).to(dtype), torch.randn(50, 3, generator=g).to(dtype)
    top, cols, fresh_flag, data = st.take_top_k_and_gather_from_main_and_fresh(
        main.to(dtype).cuda(), fresh.to(dtype).cuda(), mi.cuda(), fi.cuda(), 100, ["x"], [md.cuda()], [fd.cuda()])
    w_top, w_cols, w_fresh, w_data = select.take_top_k_and_gather(
        main.to(dtype).float().numpy(), fresh.to(dtype).float().numpy(), mi.numpy(), fi.numpy(), 100,
        md.float().numpy(), fd.float().numpy())
    assert np.array_equal(cols.cpu().numpy(), w_cols) and np.array_equal(fresh_flag.cpu().numpy(), w_fresh)
    got = top.float().cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(w_top)) and np.array_equal(got[~np.isnan(got)],
                                                                             w_top[~np.isnan(w_top)])
    assert np.array_equal(data["x"].float().cpu().numpy(), w_data)
