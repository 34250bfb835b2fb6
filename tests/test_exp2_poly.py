"""exp2_poly3 (csrc/kernels/common.cuh): the same float32 steps emulated in
numpy, with the coefficients read from the header, against exp2."""

import re
from pathlib import Path

import numpy as np

HEADER = Path(__file__).resolve().parents[1] / "csrc" / "kernels" / "common.cuh"


def _coefficients():
    body = HEADER.read_text().split("float exp2_poly3(float x) {", 1)[1].split("\n}", 1)[0]
    vals = [float(v) for v in re.findall(r"fmaf\([^;]*?(-?\d\.\d+)f\)", body)]
    # fmaf(f, c3, c2); fmaf(p, f, c1); fmaf(p, f, c0)
    c3_c2 = re.search(r"fmaf\(f, (-?\d\.\d+)f, (-?\d\.\d+)f\)", body)
    c1, c0 = vals[-2], vals[-1]
    return np.float32(c3_c2.group(1)), np.float32(c3_c2.group(2)), np.float32(c1), np.float32(c0)


def _exp2_poly3(x):
    c3, c2, c1, c0 = _coefficients()
    x = np.asarray(x, dtype=np.float32)
    xc = np.maximum(x, np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (xc + magic).astype(np.float32)
    k = t.view(np.int32) - np.int32(0x4B400000)
    f = (xc - (t - magic)).astype(np.float32)
    p = (f * c3 + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    r = (p.view(np.uint32) + (k.astype(np.uint32) << np.uint32(23))).view(np.float32)
    return np.where(x < -125.0, np.float32(0.0), r)


def test_relative_error_over_the_softmax_range():
    x = np.concatenate([np.linspace(-125, 8, 1_000_001, dtype=np.float32),
                        -np.float32(2) ** -np.arange(0, 24, dtype=np.float32)])
    rel = np.abs(_exp2_poly3(x) / np.exp2(x.astype(np.float64)) - 1)
    assert rel.max() < 1e-4, rel.max()


def test_masked_scores_give_exact_zero():
    out = _exp2_poly3(np.array([-np.inf, -1e30, -126.0, -125.5], dtype=np.float32))
    assert np.all(out == 0.0)


def _exp2_poly3_x2(x):
    """exp2_poly3_x2: same steps, exponent added as bits(t) << 23 and no
    final select (inputs below -125 are clamped)."""
    c3, c2, c1, c0 = _coefficients()
    x = np.asarray(x, dtype=np.float32)
    xc = np.maximum(x, np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (xc + magic).astype(np.float32)
    f = (xc - (t - magic)).astype(np.float32)
    p = (f * c3 + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    return (p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))).view(np.float32)


def test_pair_variant_matches_scalar_above_the_clamp():
    x = np.linspace(-125, 8, 200_001, dtype=np.float32)
    assert np.array_equal(_exp2_poly3_x2(x), _exp2_poly3(x))


def test_pair_variant_masked_scores_are_negligible():
    out = _exp2_poly3_x2(np.array([-np.inf, -1e30, -126.0], dtype=np.float32))
    assert np.all(out > 0) and np.all(out < 1e-37)
