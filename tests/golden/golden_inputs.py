"""Seeded inputs of the golden fixtures. Shared by ``make_golden.py`` (which runs
the reference on them) and the tests (which run the oracle and the kernels on
them); torch CPU generators, so every machine rebuilds the same tensors."""

from __future__ import annotations

import torch


def c1_inputs():
    """100,000 x 64 items and 256 queries, rows N(0, 1) then
    L2-normalised, seed 0, items drawn first."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(100_000, 64, generator=g)
    q = torch.randn(256, 64, generator=g)
    x = x / x.norm(dim=1, keepdim=True).clamp_min(1e-8)
    q = q / q.norm(dim=1, keepdim=True).clamp_min(1e-8)
    return q, x


def clause_inputs():
    g = torch.Generator().manual_seed(3)
    n, c, a, b = 2000, 3, 4, 16
    attrs = torch.randint(0, 8, (n, c, a), generator=g)
    attrs[torch.rand(n, c, a, generator=g) < 0.3] = -1
    q = torch.randint(0, 8, (b, c), generator=g)
    q[torch.rand(b, c, generator=g) < 0.2] = -1
    rev = torch.tensor([True, False, False])
    return attrs, rev, q


def fmkt_inputs():
    g = torch.Generator().manual_seed(5)
    b, n, d, p = 8, 3000, 64, 500
    q = torch.randn(b, d, generator=g).to(torch.float16)
    x = torch.randn(n, d, generator=g).to(torch.float16)
    pos = torch.stack([torch.randperm(n, generator=g)[:p] for _ in range(b)])
    counts = torch.randint(0, p + 1, (b,), generator=g)
    counts[0] = p
    counts[1] = 7  # fewer than k survivors: -1 / -inf tail
    return q, x, pos, counts


def oporp_inputs():
    g = torch.Generator().manual_seed(6)
    b, n, w, p = 8, 5000, 2, 300
    qb = torch.randint(-(2**63), 2**63 - 1, (b, w), generator=g, dtype=torch.int64)
    xb = torch.randint(-(2**63), 2**63 - 1, (n, w), generator=g, dtype=torch.int64)
    pos = torch.stack([torch.randperm(n, generator=g)[:p] for _ in range(b)])
    counts = torch.randint(0, p + 1, (b,), generator=g)
    counts[0] = p
    return qb, xb, pos, counts


def quantize_inputs():
    g = torch.Generator().manual_seed(7)
    x = torch.randn(64, 128, generator=g) * torch.rand(64, 1, generator=g) * 3
    x[0] = 0.0
    return x


def simhash_inputs():
    g = torch.Generator().manual_seed(8)
    return torch.randn(32, 128, generator=g)


C3_CARDS = (10, 20, 50, 100, 200, 500, 1000, 1000)


def zipf_attrs(n: int, seed: int, cards=C3_CARDS, alpha: float = 1.1):
    """BASELINE config 3 attributes: one value per attribute, value v of
    attribute c drawn with P(v) proportional to (v + 1)^-alpha over [0, card_c)."""
    g = torch.Generator().manual_seed(seed)
    cols = []
    for card in cards:
        w = (torch.arange(card, dtype=torch.float64) + 1.0) ** (-alpha)
        cols.append(torch.multinomial(w, n, replacement=True, generator=g))
    return torch.stack(cols, dim=1).to(torch.int64)


BLOOM_EXPRESSIONS = [
    "0:0",
    "1:3 OR 2:7",
    "0:1 AND 3:2",
    "NOT 0:0",
    "(4:5 OR 5:1) AND 0:2",
    "6:0 OR 7:0 OR 2:1",
    "1:0 AND NOT 2:0",
    "3:10 OR (0:4 AND 1:1)",
    "5:0 AND 6:1 AND 7:2",
    "NOT (0:0 OR 1:0)",
    "2:3",
    "7:999 OR 0:9",
]
