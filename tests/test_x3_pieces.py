"""The arithmetic GSV_MODE_FP32_TC rests on, checked on the CPU.

Every decoder activation and weight is held as three bf16 pieces: piece 0 the
round-to-nearest-even bf16 of the fp32 value v, piece 1 that of v - piece 0,
piece 2 that of what is left (the epilogue's store_x3, the relayout's st_x3
and the weight packer all split this way).  A normal fp32 value has 24
significant bits and each piece takes the next 8, so the pieces sum back to v
exactly.  A product x * w is formed from the six piece products
X0W0 + X0W1 + X1W0 + X0W2 + X1W1 + X2W0; the dropped X1W2, X2W1, X2W2 are
below 2^-23 of |x w| together.
"""
from __future__ import annotations

import numpy as np
import torch


def _pieces(v: np.ndarray):
    r = torch.from_numpy(v.astype(np.float32))
    out = []
    for _ in range(3):
        p = r.to(torch.bfloat16)
        out.append(p.to(torch.float32))
        r = r - out[-1]
    return [p.numpy() for p in out]


def _values(n, seed, lo=-60, hi=60):
    rng = np.random.default_rng(seed)
    m = rng.uniform(1.0, 2.0, n)
    e = rng.integers(lo, hi, n)
    s = rng.choice([-1.0, 1.0], n)
    return (s * m * np.exp2(e)).astype(np.float32)


def test_three_pieces_sum_back_exactly():
    v = _values(200_000, 1)
    p0, p1, p2 = _pieces(v)
    assert np.array_equal((p0 + p1) + p2, v)  # the order every reader of the pieces uses
    assert np.array_equal(p0 + (p1 + p2), v)
    # each piece holds at most 8 significant bits
    for p in (p0, p1, p2):
        nz = p[p != 0]
        mant = (nz.view(np.uint32) & 0x7FFFFF)
        assert not np.any(mant & 0xFFFF)


def test_zero_and_exact_bf16_values_have_zero_remainders():
    v = np.array([0.0, -0.0, 1.0, -2.5, 0.1015625, 3.0e38], np.float32)
    p0, p1, p2 = _pieces(v)
    exact = np.array([True, True, True, True, True, False])
    assert np.array_equal((p0 + p1) + p2, v)
    assert not p1[exact].any() and not p2[exact].any()


def test_six_piece_products_reach_fp32_accuracy():
    x, w = _values(100_000, 2, -20, 20), _values(100_000, 3, -20, 20)
    x0, x1, x2 = (p.astype(np.float64) for p in _pieces(x))
    w0, w1, w2 = (p.astype(np.float64) for p in _pieces(w))
    six = x0 * w0 + x0 * w1 + x1 * w0 + x0 * w2 + x1 * w1 + x2 * w0
    exact = x.astype(np.float64) * w.astype(np.float64)
    rel = np.abs(six - exact) / np.abs(exact)
    assert rel.max() <= 2.0 ** -23
    # a bf16 x bf16 product is exact in fp32 (8 x 8 significant bits)
    prods = (x0 * w1).astype(np.float32).astype(np.float64)
    assert np.array_equal(prods, x0 * w1)
