"""Int8 scoring + top-k against the CPU oracle: int32 dots
are exact, the dequant order is the reference's, so ids and scores are
bit-exact, ties toward the lower id."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import knn
from tests.helpers import assert_topk_exact

pytestmark = pytest.mark.gpu


def _items(n, d, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g)
    scales = x.abs().amax(dim=1).clamp_min(1e-8) / 127.0
    codes = torch.round(x / scales[:, None]).clamp(-127, 127).to(torch.int8)
    return codes, scales.to(torch.float32)


@pytest.mark.parametrize("b,n,d,k", [(64, 20_000, 256, 100), (300, 50_000, 256, 50), (130, 7_777, 128, 100),
                                     (1024, 300_000, 256, 100)])
def test_int8_topk_bit_exact(b, n, d, k):
    from retrieve_b200 import ops

    codes, scales = _items(n, d, seed=n)
    q = torch.randn(b, d, generator=torch.Generator().manual_seed(b))
    ids, scores = ops.int8_topk(q.cuda(), codes.cuda(), scales.cuda(), k)
    ref_ids, ref_scores = knn.int8_topk(q.numpy(), codes.numpy(), scales.numpy(), k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)


def test_int8_global_scale_equals_silvertorch_full_probe():
    """With one global item scale the ranking is the raw int32 dot's, as in
    SilverTorch's st::search with every cluster probed."""
    from retrieve_b200 import ops

    b, n, d, k = 96, 30_000, 256, 100
    g = torch.Generator().manual_seed(9)
    x = torch.randn(n, d, generator=g)
    gscale = float(x.abs().max() / 127.0)
    codes = torch.round(x / gscale).clamp(-127, 127).to(torch.int8)
    q = torch.randn(b, d, generator=g)
    ids, scores = ops.int8_topk(q.cuda(), codes.cuda(), torch.full((n,), gscale).cuda(), k)
    ref_ids, ref_scores = knn.silvertorch_fullprobe(q.numpy(), codes.numpy(), gscale, k)
    assert_topk_exact(ids.cpu().numpy(), scores.cpu().numpy(), ref_ids, ref_scores)
