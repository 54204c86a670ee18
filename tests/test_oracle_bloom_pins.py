"""Pins the Bloom / predicate oracle to the reference's own SilverTorch CPU ops
(fixtures from tests/golden/make_golden_bloom.py). CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import bloom, predicate
from tests.golden import golden_inputs as gi

G = np.load(Path(__file__).resolve().parent / "golden" / "golden_bloom.npz")


def test_item_words_equal_reference_bloom_build():
    n = int(G["n"])
    ref_words = bloom.transpose_reference_bundle(G["bloom_index"], n)
    assert np.array_equal(bloom.item_words(G["attrs"], k=3), ref_words)


def test_predicate_on_bloom_equals_reference_search():
    n = int(G["n"])
    words = bloom.transpose_reference_bundle(G["bloom_index"], n)
    masks = np.unpackbits(G["masks"], axis=1)[:, :n].astype(bool)
    for i, expr in enumerate(gi.BLOOM_EXPRESSIONS):
        got = predicate.eval_items(predicate.parse(expr), words=words, k=3, n_stored=7)
        assert np.array_equal(got, masks[i]), expr


def test_bloom_has_no_false_negatives():
    n = int(G["n"])
    words = bloom.transpose_reference_bundle(G["bloom_index"], n)
    attrs = G["attrs"]
    for expr in gi.BLOOM_EXPRESSIONS:
        if "NOT" in expr:
            continue
        ast = predicate.parse(expr)
        exact = predicate.eval_items(ast, attrs=attrs)
        approx = predicate.eval_items(ast, words=words, k=3, n_stored=7)
        assert not (exact & ~approx).any(), expr


def test_murmur_is_deterministic_and_spreads():
    h = {bloom.murmur_hash3_2x64(c, v, s) for c in range(4) for v in range(50) for s in range(3)}
    assert len(h) == 600
