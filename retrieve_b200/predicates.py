"""Attribute predicates for the filtered dense search: building the per-query
term programs the kernels evaluate (``rb_pred_term``, include/retrieve_b200.h).

Two sources, the two filter front-ends of the reference:
  * LiNR's exact clause filter: ``query_clause_attrs [B, C]`` (``-1`` =
    inactive clause) and ``clause_is_reverse [C]`` — AND over the active clauses
    of "the item's clause c holds the value", negated for reverse clauses
    (retrieve/src/retrieve/functional.py:173-185).
  * SilverTorch's query DSL: ``"1:100 AND (2:200 OR NOT 3:300)"``
    (silvertorch/silvertorch/ops/csrc/EXPRESSION_SYNTAX.md; NOT > AND > OR,
    parentheses, ``& | !``, the empty string matches everything). Expressions
    are rewritten into conjunctive normal form (AND of ORs of possibly negated
    terms), at most 8 terms.

Each term also carries its 64-bit Bloom mask: the first ``k`` distinct
positions ``murmur_hash3_2x64(clause, value, seed) % 64`` among the first
``n_stored_hashes`` seeds (silvertorch bloom_index_util.cuh:61-107 and
bloom_index_search_cuda.cu:304-349: a term may test fewer than k bits). Query
preparation is host work outside the timed search, as in the reference
(``SilverTorch.prepare_queries``, retrieve/src/retrieve/modules/silvertorch.py:258-289).
"""

from __future__ import annotations

import re
from dataclasses import dataclass

import numpy as np
import torch

MAX_TERMS = 8
TERM_DTYPE = np.dtype([("value", "<i8"), ("bloom_mask", "<u8"), ("clause", "<i4"), ("flags", "<i4")])
_M64 = (1 << 64) - 1


def _rotl(x: int, r: int) -> int:
    return ((x << r) | (x >> (64 - r))) & _M64


def _fmix(k: int) -> int:
    k ^= k >> 33
    k = (k * 0xFF51AFD7ED558CCD) & _M64
    k ^= k >> 33
    k = (k * 0xC4CEB9FE1A85EC53) & _M64
    return k ^ (k >> 33)


def murmur_hash3_2x64(x: int, y: int, seed: int) -> int:
    """MurmurHash3 x64-128 (Appleby) of the 16-byte key (x, y), halves XOR-ed."""
    c1, c2 = 0x87C37B91114253D5, 0x4CF5AD432745937F
    h1 = h2 = seed & _M64
    h1 ^= (_rotl((x & _M64) * c1 & _M64, 31) * c2) & _M64
    h1 = (_rotl(h1, 27) + h2) & _M64
    h1 = (h1 * 5 + 0x52DCE729) & _M64
    h2 ^= (_rotl((y & _M64) * c2 & _M64, 33) * c1) & _M64
    h2 = (_rotl(h2, 31) + h1) & _M64
    h2 = (h2 * 5 + 0x38495AB5) & _M64
    h1 ^= 16
    h2 ^= 16
    h1 = (h1 + h2) & _M64
    h2 = (h2 + h1) & _M64
    h1, h2 = _fmix(h1), _fmix(h2)
    h1 = (h1 + h2) & _M64
    h2 = (h2 + h1) & _M64
    return h1 ^ h2


def bloom_term_mask(clause: int, value: int, k: int = 3, n_stored_hashes: int = 7) -> int:
    mask, got = 0, 0
    for seed in range(n_stored_hashes):
        if got >= k:
            break
        bit = 1 << (murmur_hash3_2x64(clause, value, seed) % 64)
        if not mask & bit:
            mask |= bit
            got += 1
    return mask


# --- the DSL ----------------------------------------------------------------
_TOK = re.compile(r"\s*(\(|\)|!|&|\||AND\b|OR\b|NOT\b|-?\d+:-?\d+(?::[-+.\deE]+)?)")


def _parse(expr: str):
    toks, pos = [], 0
    s = expr.strip()
    while pos < len(s):
        m = _TOK.match(s, pos)
        if not m:
            raise ValueError(f"cannot parse expression {expr!r} at {s[pos:]!r}")
        toks.append(m.group(1))
        pos = m.end()
    if not toks:
        return None
    i = 0

    def peek():
        return toks[i] if i < len(toks) else None

    def nxt():
        nonlocal i
        i += 1
        return toks[i - 1]

    def e_or():
        node = e_and()
        while peek() in ("OR", "|"):
            nxt()
            node = ("or", node, e_and())
        return node

    def e_and():
        node = e_not()
        while peek() in ("AND", "&"):
            nxt()
            node = ("and", node, e_not())
        return node

    def e_not():
        if peek() in ("NOT", "!"):
            nxt()
            return ("not", e_not())
        t = nxt()
        if t == "(":
            node = e_or()
            if nxt() != ")":
                raise ValueError(f"unbalanced parentheses in {expr!r}")
            return node
        c, v = t.split(":")[:2]
        return ("lit", int(c), int(v), False)

    node = e_or()
    if i != len(toks):
        raise ValueError(f"trailing tokens in {expr!r}")
    return node


def _nnf(node, neg=False):
    kind = node[0]
    if kind == "lit":
        return ("lit", node[1], node[2], node[3] != neg)
    if kind == "not":
        return _nnf(node[1], not neg)
    a, b = _nnf(node[1], neg), _nnf(node[2], neg)
    op = node[0] if not neg else ("or" if node[0] == "and" else "and")
    return (op, a, b)


def _cnf(node) -> list[frozenset]:
    if node[0] == "lit":
        return [frozenset([node[1:]])]
    a, b = _cnf(node[1]), _cnf(node[2])
    if node[0] == "and":
        return a + b
    return [x | y for x in a for y in b]


def expression_to_cnf(expr: str) -> list[list[tuple[int, int, bool]]]:
    """Clauses (OR-groups) of literals ``(clause, value, negated)``."""
    ast = _parse(expr)
    if ast is None:
        return []
    out, seen = [], set()
    for cl in _cnf(_nnf(ast)):
        if any((c, v, not n) in cl for (c, v, n) in cl):
            continue  # tautology (x OR NOT x)
        if cl not in seen:
            seen.add(cl)
            out.append(sorted(cl))
    return out


@dataclass
class Predicates:
    """Per-query term programs on the device: ``terms`` [B, 8 * 24] uint8
    (``rb_pred_term``) and ``n_terms`` [B] int32."""

    terms: torch.Tensor
    n_terms: torch.Tensor

    def to(self, device) -> Predicates:
        return Predicates(self.terms.to(device), self.n_terms.to(device))


def _pack(rows: list[list[list[tuple[int, int, bool]]]], k: int, n_stored: int) -> Predicates:
    arr = np.zeros((len(rows), MAX_TERMS), dtype=TERM_DTYPE)
    n = np.zeros(len(rows), dtype=np.int32)
    cache: dict[tuple[int, int], int] = {}
    for r, clauses in enumerate(rows):
        if len(clauses) > MAX_TERMS:
            raise ValueError(f"predicate of row {r} has {len(clauses)} OR-groups; at most {MAX_TERMS}")
        t = 0
        for g, clause in enumerate(clauses):
            for c, v, neg in clause:
                if t >= MAX_TERMS:
                    raise ValueError(f"predicate of row {r} needs more than {MAX_TERMS} terms")
                key = (int(c), int(v))
                if key not in cache:
                    cache[key] = bloom_term_mask(key[0], key[1], k, n_stored)
                arr[r, t] = (v, cache[key], c, g | (8 if neg else 0))
                t += 1
        n[r] = t
    return Predicates(torch.from_numpy(arr.view(np.uint8).reshape(len(rows), -1).copy()), torch.from_numpy(n))


def from_expressions(expressions: list[str], *, k: int = 3, n_stored_hashes: int = 7) -> Predicates:
    return _pack([expression_to_cnf(e) for e in expressions], k, n_stored_hashes)


def from_clause_attrs(query_clause_attrs: torch.Tensor, clause_is_reverse: torch.Tensor | None = None, *,
                      k: int = 3, n_stored_hashes: int = 7) -> Predicates:
    """LiNR's exact-filter queries: AND over active clauses (``-1`` = inactive),
    each negated when its clause is a reverse clause."""
    qa = query_clause_attrs.to("cpu", torch.int64).numpy()
    rev = (np.zeros(qa.shape[1], dtype=bool) if clause_is_reverse is None
           else clause_is_reverse.to("cpu").numpy().astype(bool))
    rows = [[[(c, int(v), bool(rev[c]))] for c, v in enumerate(row) if v != -1] for row in qa]
    return _pack(rows, k, n_stored_hashes)


__all__ = ["Predicates", "bloom_term_mask", "expression_to_cnf", "from_clause_attrs", "from_expressions",
           "murmur_hash3_2x64"]
