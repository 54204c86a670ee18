"""An IVF index built and searched end to end by the library's own parts, the way SilverTorch's
builder and layer chain the reference's ops (retrieve/src/retrieve/modules/silvertorch.py): k-means
lists (``retrieve_b200.kmeans``), the cluster-sorted table and its global int8 scale
(``quantize_int8_global``), SilverTorch's bloom index over the sorted attributes, plans from the
library's parser, then ``st::search`` on the row and grouped scorers — each result checked against
the restatements on the same built arrays (and the k-means against the reference's fixture)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ivf
from oracle import kmeans as okm

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden_kmeans.npz")


@pytest.mark.gpu
@pytest.mark.parametrize("grouped", [False, True])
def test_built_index_searches_like_the_restatement(grouped):
    import retrieve_b200.st  # noqa: F401  (registers torch.ops.st)
    from retrieve_b200 import st
    from retrieve_b200.kmeans import KMeans
    from retrieve_b200.quantize import quantize_int8_global

    x = torch.from_numpy(GOLDEN["x"]).cuda()
    n, d = x.shape
    n_lists = 8
    centroids, assign = KMeans(n_lists, 5, seed=3, init="kmeans++").fit(x)
    want_c, want_a = okm.fit(GOLDEN["x"], n_lists, 5, seed=3, init="kmeans++")
    assert np.array_equal(centroids.cpu().numpy(), want_c) and np.array_equal(assign.cpu().numpy(), want_a)

    perm = torch.sort(assign, stable=True).indices  # sorted position -> item id
    sizes = torch.bincount(assign, minlength=n_lists)
    offsets = torch.zeros(n_lists + 1, dtype=torch.int64, device="cuda")
    offsets[1:] = sizes.cumsum(0)
    codes, gs = quantize_int8_global(x, rows=perm)
    gst = torch.tensor(gs, dtype=torch.float32, device="cuda")

    rng = np.random.default_rng(5)
    b, n_probe, k = 12, 3, 20
    q = torch.from_numpy(rng.standard_normal((b, d)).astype(np.float32)).cuda()
    probe = torch.topk(q @ centroids.t(), n_probe, dim=1).indices
    width = int(sizes[probe].sum(1).max())

    # attributes in sorted order, their bloom index, one AND expression per query
    attrs = rng.integers(0, 6, (n, 2, 2))
    attrs[rng.random((n, 2, 2)) < 0.3] = -1
    sorted_attrs = attrs[perm.cpu().numpy()]
    fid, foff, fval = ivf.attrs_to_features(sorted_attrs)
    index, boff = st.bloom_index_build(*(torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (fid, foff, fval)),
                                       10.0, 3)
    exprs = [f"0:{rng.integers(0, 6)}" + (f" AND 1:{rng.integers(0, 6)}" if i % 2 else "") for i in range(b)]
    stack, (data, plan_off) = torch.ops.st.parse_expression_query_batch(exprs, torch.ones(b), 7, True, 5)
    blob = torch.from_numpy(ivf.plan_blob(data.numpy(), plan_off.numpy(), b)).cuda()

    fn = st.search_grouped if grouped else st.search_rows
    args = (q, probe, offsets, sizes, codes, perm, gst, k, width)
    ids, scores = fn(*args)
    host = [t.cpu().numpy() for t in (q, probe, offsets, sizes, codes, perm)]
    want = ivf.search(*host, gst.cpu().numpy(), k, width)
    assert np.array_equal(ids.cpu().numpy(), want[0]) and np.array_equal(scores.cpu().numpy(), want[1])

    ids_b, scores_b = fn(*args, bloom_index=index, bloom_bundle_b_offsets=boff, plans=blob, plan_count=b,
                         max_stack_size=stack, bloom_k=3, hash_k=7)
    masks = np.stack([ivf.bloom_plan_mask(index.cpu().numpy(), boff.cpu().numpy(), data.numpy(), plan_off.numpy(),
                                          p, 3, 7, n) for p in range(b)])
    want_b = ivf.search(*host, gst.cpu().numpy(), k, width, filtering_bit_mask=ivf.pack_mask_high_first(masks))
    assert np.array_equal(ids_b.cpu().numpy(), want_b[0]) and np.array_equal(scores_b.cpu().numpy(), want_b[1])
