"""The fused output stages' arithmetic (ork_i8_mm_run_out8 / _out16 / _ewmul, ork_i8_npu_ewmul) in the
oracle, pinned without a GPU.

The reference's model of its NPU requant stage (examples/test_mm_i8_out8.c:24-33) rounds v * mult / 2^shift
half to even; its comment lists the silicon-verified ties 30.5 -> 30, 39.5 -> 40, -7.5 -> -8, 0.5 -> 0 and
clamps to [-128, 127]. The oracle (oracle/ork_oracle.c orc_requant) is checked against those ties and
against an independent exact model here (Python Fractions: round() on a Fraction is round-half-even).
"""
from fractions import Fraction

import numpy as np

import oracle_ffi as of


def _exact(acc, mult, shift, bits=8, g=None):
    lo, hi = (-32768, 32767) if bits == 16 else (-128, 127)
    out = []
    for i, a in enumerate(np.asarray(acc, np.int64).ravel()):
        v = int(a) * mult * (int(g.ravel()[i]) if g is not None else 1)
        q = round(Fraction(v, 1 << shift))
        out.append(min(hi, max(lo, q)))
    return np.array(out, np.int64).reshape(np.shape(acc))


def test_reference_ties_round_half_to_even():
    # acc * mult / 2^shift = x.5 exactly: with mult = 1, shift = 1, acc = 2x + 1
    acc = np.array([61, 79, -15, 1, -1, 3, -3], np.int32)  # 30.5 39.5 -7.5 0.5 -0.5 1.5 -1.5
    got = of.requant(acc, 1, 1)
    assert got.tolist() == [30, 40, -8, 0, 0, 2, -2]


def test_identity_gain_is_clamp():
    acc = np.array([0, 1, -1, 127, 128, -128, -129, 100000, -100000], np.int32)
    assert of.requant(acc, 0x4000, 14).tolist() == [0, 1, -1, 127, 127, -128, -128, 127, -128]
    assert of.requant(acc, 0x4000, 14, bits=16).tolist() == [0, 1, -1, 127, 128, -128, -129, 32767, -32768]


def test_random_against_exact_model():
    rng = np.random.default_rng(3)
    for mult, shift in [(0x4000, 14), (0x2000, 14), (0x1000, 15), (0x2AB0, 15), (7, 0), (1, 20), (0x7FFF, 31)]:
        acc = rng.integers(-(1 << 24), 1 << 24, size=2000).astype(np.int32)
        for bits in (8, 16):
            assert np.array_equal(of.requant(acc, mult, shift, bits), _exact(acc, mult, shift, bits)), (mult, shift)
        g = rng.integers(-128, 128, size=acc.shape).astype(np.int8)
        assert np.array_equal(of.requant(acc, mult, shift, 8, g), _exact(acc, mult, shift, 8, g)), (mult, shift)


def test_ewmul_extremes():
    # the largest magnitudes a full-K int8 matmul (K <= 4096) can produce, times G = -128, times 0x7fff
    acc = np.array([4096 * 128 * 128, -4096 * 128 * 127], np.int32)
    g = np.array([-128, -128], np.int8)
    assert np.array_equal(of.requant(acc, 0x7FFF, 31, 8, g), _exact(acc, 0x7FFF, 31, 8, g))
