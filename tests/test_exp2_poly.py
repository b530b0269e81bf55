"""The polynomial 2^x that the chunked-prefill softmax evaluates on the FMA pipe for a third of its
exponentials (exp2_poly2 in csrc/pkv_common.cuh), emulated bit for bit in float32 on the host from the
constants in the source: relative error against exact 2^x at most 2^-13.5 (the Remez bound of the
polynomial is 7.48e-5), below half a unit in the last place of the 16-bit probabilities it feeds; the
range reduction is exact (integer x give the polynomial's value at 0 times an exact power of two);
-inf and anything below -125 give a tiny normal number instead of 0."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "qwen3.6-2080ti_b200" / "csrc" / "pkv_common.cuh"


def _coefficients() -> list[np.float32]:
    text = SRC.read_text()
    out = []
    for k in range(4):
        m = re.search(rf"kExp2Poly{k} = ([0-9a-fx.p+-]+)f", text)
        assert m, k
        out.append(np.float32(float.fromhex(m.group(1))))
    return out


def _fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x: np.ndarray) -> np.ndarray:
    c = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic).astype(np.float32)).astype(np.float32)
    p = _fma32(f, np.full_like(f, c[3]), np.full_like(f, c[2]))
    p = _fma32(p, f, np.full_like(f, c[1]))
    p = _fma32(p, f, np.full_like(f, c[0]))
    bits = (t.view(np.uint32).astype(np.uint64) << np.uint64(23)) + p.view(np.uint32).astype(np.uint64)
    return (bits & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)


def test_relative_error_over_the_softmax_range() -> None:
    x = np.concatenate([np.linspace(-125.0, 12.0, 2_000_001, dtype=np.float32),
                        np.float32(-0.5) + np.arange(-2000, 2000, dtype=np.float32) * np.float32(2.0 ** -12)])
    got = exp2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() <= 2.0 ** -13.5, (rel.max(), x[np.argmax(rel)])


def test_range_reduction_is_exact_on_integers() -> None:
    c0 = _coefficients()[0]
    j = np.arange(-125, 120, dtype=np.float32)
    np.testing.assert_array_equal(exp2_poly(j), (np.float64(c0) * np.exp2(j.astype(np.float64))).astype(np.float32))


def test_masked_scores_give_a_tiny_normal_value() -> None:
    out = exp2_poly(np.array([-np.inf, -1e30, -126.0, -125.0], dtype=np.float32))
    assert np.all(out > 0) and np.all(out < 2.0 ** -124)
    assert np.all(np.isfinite(out))
