"""The float dot products of SilverTorch's CUDA scorer (silvertorch/ops/csrc/simple_index_mm.cuh
:41-56, 96-151, 160-300) restated on the CPU with exact rounding. Test infrastructure: only the
tests use it, as the checker.

Per doc one fused multiply-add chain per block of ``unit`` elements, each step rounded once to
the format (round to nearest, ties to even): fp32 in one accumulator; fp16 / bf16 in a packed
pair, even elements in one half and odd in the other. Blocks are added in order onto zero (a row
of at most 256 bytes is one block taken as it is; a single 384-byte block is still added onto
zero, which turns a -0 into +0) and the pair's halves added last. ``unit`` is the whole row
when it fits 256 bytes, else 256 bytes' worth of elements when that divides D, else 384 bytes'
worth (simple_index_mm.cuh:237-300).

Every step is computed exactly: the product of two format values is exact in float64, and the
sum with the accumulator is checked exact by TwoSum; when it is not, the step is redone in
rational arithmetic, so no result is rounded twice.
"""

from __future__ import annotations

import math
from fractions import Fraction

import numpy as np

# (mantissa bits including the implicit one, smallest normal exponent, largest exponent)
FORMATS = {"fp32": (24, -126, 127), "fp16": (11, -14, 15), "bf16": (8, -126, 127)}
ELEM_BYTES = {"fp32": 4, "fp16": 2, "bf16": 2}


def _round(value, fmt: str) -> float:
    """``value`` (a float64 or a Fraction, exact) rounded once to ``fmt``, as a float."""
    p, emin, emax = FORMATS[fmt]
    if value == 0:
        return 0.0
    neg = value < 0
    a = -value if neg else value
    if isinstance(a, Fraction):
        e = a.numerator.bit_length() - a.denominator.bit_length()
        if Fraction(2) ** e > a:
            e -= 1
        if Fraction(2) ** (e + 1) <= a:
            e += 1
        shift = max(e, emin) - p + 1
        q = a / Fraction(2) ** shift
        n = q.numerator // q.denominator
        rem = q - n
        if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2 == 1):
            n += 1
        v = math.ldexp(float(n), shift)
    else:
        _, e2 = math.frexp(a)
        shift = max(e2 - 1, emin) - p + 1
        v = math.ldexp(float(round(math.ldexp(a, -shift))), shift)  # round(): ties to even, exact here
    if v >= math.ldexp(1.0, emax + 1):
        v = math.inf
    return -v if neg else v


def _add_exact(x: float, y: float, fmt: str) -> float:
    s = x + y
    if math.isfinite(s):
        bv = s - x
        err = (x - (s - bv)) + (y - bv)  # TwoSum: s + err == x + y exactly
        if err == 0:
            if s == 0:
                return -0.0 if (math.copysign(1, x) < 0 and math.copysign(1, y) < 0) else 0.0
            return _round(s, fmt)
    return _round(Fraction(x) + Fraction(y), fmt)


def fma(a: float, b: float, c: float, fmt: str) -> float:
    """``a * b + c`` rounded once to ``fmt`` (a, b, c values of the format)."""
    prod = a * b  # exact in float64 for all three formats
    if prod == 0 and c == 0:
        return -0.0 if (math.copysign(1, prod) < 0 and math.copysign(1, c) < 0) else 0.0
    return _add_exact(prod, c, fmt)


def add(a: float, b: float, fmt: str) -> float:
    return _add_exact(a, b, fmt)


def unit(d: int, fmt: str) -> int:
    """The chain length for rows of ``d`` elements (0: no kernel for that ``d``)."""
    eb = ELEM_BYTES[fmt]
    if d % (16 // eb):
        return 0
    if d * eb <= 256:
        return d
    if d % (256 // eb) == 0:
        return 256 // eb
    if d % (384 // eb) == 0:
        return 384 // eb
    return 0


def dot(x_row, q_row, fmt: str) -> float:
    """The scorer's dot of one doc row with one query row (values already in ``fmt``)."""
    x = [float(v) for v in np.asarray(x_row, dtype=np.float64)]
    q = [float(v) for v in np.asarray(q_row, dtype=np.float64)]
    d = len(x)
    u = unit(d, fmt)
    if u == 0:
        raise ValueError(f"no {fmt} chain for D = {d}")
    pair = fmt != "fp32"

    def block(lo):
        if not pair:
            acc = 0.0
            for i in range(lo, lo + u):
                acc = fma(x[i], q[i], acc, fmt)
            return (acc,)
        ev = od = 0.0
        for i in range(lo, lo + u, 2):
            ev = fma(x[i], q[i], ev, fmt)
            od = fma(x[i + 1], q[i + 1], od, fmt)
        return (ev, od)

    if d * ELEM_BYTES[fmt] <= 256:  # one block, taken as it is
        acc = block(0)
    else:  # blocks added onto zero, even when one block (384 bytes) is the whole row
        acc = (0.0, 0.0) if pair else (0.0,)
        for lo in range(0, d, u):
            blk = block(lo)
            acc = tuple(add(a, b, fmt) for a, b in zip(acc, blk))
    return add(acc[0], acc[1], fmt) if pair else acc[0]


def to_format(x, fmt: str) -> np.ndarray:
    """float64 values rounded to ``fmt`` (elementwise, once)."""
    flat = np.asarray(x, dtype=np.float64).reshape(-1)
    return np.array([_round(float(v), fmt) for v in flat], dtype=np.float64).reshape(np.shape(x))
