"""Host-side predicate programs (retrieve_b200.predicates) against the oracle:
the CNF rewrite of each DSL expression selects the same items as direct
evaluation of its syntax tree, Bloom term masks equal the oracle's, and LiNR
clause queries equal the exact clause filter. CPU only."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bloom, filters, predicate
from retrieve_b200 import predicates as P
from tests.golden import golden_inputs as gi


def _eval_cnf(cnf, attrs):
    out = np.ones(attrs.shape[0], dtype=bool)
    for clause in cnf:
        any_ = np.zeros(attrs.shape[0], dtype=bool)
        for c, v, neg in clause:
            m = (attrs[:, c, None] == v).any(axis=1) if attrs.ndim == 2 else (attrs[:, c, :] == v).any(axis=1)
            any_ |= ~m if neg else m
        out &= any_
    return out


EXTRA = ["", "NOT NOT 1:2", "!(0:1 & 1:1) | 2:2", "(0:0 OR 1:1) AND (2:2 OR 3:3)", "0:5 OR NOT 0:5"]


@pytest.mark.parametrize("expr", gi.BLOOM_EXPRESSIONS + EXTRA)
def test_cnf_rewrite_selects_the_same_items(expr):
    attrs = gi.zipf_attrs(3000, seed=5).numpy()
    ref = predicate.eval_items(predicate.parse(expr), attrs=attrs)
    assert np.array_equal(_eval_cnf(P.expression_to_cnf(expr), attrs), ref)


def test_bloom_term_masks_equal_oracle():
    for c in range(8):
        for v in range(40):
            assert P.bloom_term_mask(c, v, 3, 7) == bloom.term_mask(c, v, 3, 7)
            assert P.murmur_hash3_2x64(c, v, 2) == bloom.murmur_hash3_2x64(c, v, 2)


def test_clause_attr_queries_equal_exact_filter():
    g = torch.Generator().manual_seed(2)
    attrs = torch.randint(0, 6, (500, 3, 2), generator=g)
    attrs[torch.rand(500, 3, 2, generator=g) < 0.3] = -1
    q = torch.randint(0, 6, (20, 3), generator=g)
    q[torch.rand(20, 3, generator=g) < 0.3] = -1
    rev = torch.tensor([False, True, False])
    preds = P.from_clause_attrs(q, rev)
    arr = preds.terms.numpy().view(P.TERM_DTYPE).reshape(20, P.MAX_TERMS)
    ref = filters.clause_mask(attrs.numpy(), rev.numpy(), q.numpy())
    for r in range(20):
        cnf = [[(int(t["clause"]), int(t["value"]), bool(t["flags"] & 8))] for t in arr[r, : preds.n_terms[r]]]
        assert np.array_equal(_eval_cnf(cnf, attrs.numpy()), ref[r])


def test_too_many_terms_rejected():
    with pytest.raises(ValueError):
        P.from_expressions([" OR ".join(f"{i % 8}:{i}" for i in range(9))])
