"""Attribute predicates restated for the oracle (test infrastructure).

Grammar of the reference's query DSL (silvertorch/silvertorch/ops/csrc/
EXPRESSION_SYNTAX.md): terms ``id:value``, ``NOT``/``!`` > ``AND``/``&`` >
``OR``/``|``, parentheses; the empty expression matches everything
(expression_query_parser.cpp:400-405). A term ``c:v`` matches an item when:
  * exact: some value of the item's clause c equals v (functional.py:173-185);
  * bloom: the item's 64-bit word has every search position of (c, v) set
    (oracle/bloom.py).
Evaluated directly on the syntax tree (no normal-form rewriting).
"""

from __future__ import annotations

import re

import numpy as np

from oracle import bloom

_TOKEN = re.compile(r"\s*(\(|\)|!|&|\||AND\b|OR\b|NOT\b|-?\d+:-?\d+(?::[-+.\deE]+)?)")


def tokenize(expr: str) -> list[str]:
    out, pos = [], 0
    expr = expr.strip()
    while pos < len(expr):
        m = _TOKEN.match(expr, pos)
        if not m:
            raise ValueError(f"bad expression near {expr[pos:]!r}")
        out.append(m.group(1))
        pos = m.end()
    return out


def parse(expr: str):
    toks = tokenize(expr)
    if not toks:
        return ("all",)
    pos = 0

    def peek():
        return toks[pos] if pos < len(toks) else None

    def take():
        nonlocal pos
        pos += 1
        return toks[pos - 1]

    def p_or():
        xs = [p_and()]
        while peek() in ("OR", "|"):
            take()
            xs.append(p_and())
        return xs[0] if len(xs) == 1 else ("or", xs)

    def p_and():
        xs = [p_not()]
        while peek() in ("AND", "&"):
            take()
            xs.append(p_not())
        return xs[0] if len(xs) == 1 else ("and", xs)

    def p_not():
        if peek() in ("NOT", "!"):
            take()
            return ("not", p_not())
        return p_atom()

    def p_atom():
        t = take()
        if t == "(":
            x = p_or()
            if take() != ")":
                raise ValueError("unbalanced parentheses")
            return x
        c, v = t.split(":")[:2]
        return ("term", int(c), int(v))

    ast = p_or()
    if pos != len(toks):
        raise ValueError("trailing tokens")
    return ast


def eval_items(ast, *, attrs=None, words=None, k=3, n_stored=7) -> np.ndarray:
    """Vectorised evaluation over items: exact when ``attrs`` ([N, C] or
    [N, C, A] int64) is given, bloom when ``words`` ([N] uint64) is given."""
    n = attrs.shape[0] if attrs is not None else words.shape[0]
    if attrs is not None and attrs.ndim == 2:
        attrs = attrs[:, :, None]

    def ev(node):
        kind = node[0]
        if kind == "all":
            return np.ones(n, dtype=bool)
        if kind == "term":
            _, c, v = node
            if attrs is not None:
                return (attrs[:, c, :] == v).any(axis=1)
            m = np.uint64(bloom.term_mask(c, v, k, n_stored))
            return (words & m) == m
        if kind == "not":
            return ~ev(node[1])
        if kind == "and":
            out = np.ones(n, dtype=bool)
            for x in node[1]:
                out &= ev(x)
            return out
        out = np.zeros(n, dtype=bool)
        for x in node[1]:
            out |= ev(x)
        return out

    return ev(ast)
