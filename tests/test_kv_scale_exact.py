# SPDX-License-Identifier: Apache-2.0
"""The INT8 KV writer's division-free row scale is the IEEE quotient.

The kernel (row_scale in glm-5.3-kernels_b200/csrc/titan_kv.cu) computes
scale = max(amax / 127, 1e-12) (kernels/titan_kv.py:16) as
y0 = fl(amax * c), c = fl(1/127), then y = fma(fma(-y0, 127, amax), c, y0)
(one FMA residual correction, Markstein 1990).  amax is the magnitude of a
bf16 value, so the claim is checked exhaustively: for all 32,640 non-negative
finite bf16 values, with exact rational arithmetic and round-to-nearest-even
to float32 standing in for the GPU's fmul / fma.
"""
import struct
from fractions import Fraction

HALF = Fraction(1, 2)


def f32(x):
    """Nearest float32 (ties to even) of an exact rational, as a Fraction."""
    if x == 0:
        return Fraction(0)
    sign = -1 if x < 0 else 1
    x = abs(x)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    if Fraction(2) ** e > x:
        e -= 1
    e = max(e, -126)                      # below 2^-126 the quantum is fixed at 2^-149
    quantum = Fraction(2) ** (e - 23)
    n = x / quantum
    whole = n.numerator // n.denominator
    rem = n - whole
    if rem > HALF or (rem == HALF and whole % 2):
        whole += 1
    return sign * whole * quantum


def test_f32_rounding_helper():
    for v in (1.0, 0.1, 1e-40, 3.4e38, 127.0 / 3):
        assert float(f32(Fraction(v))) == struct.unpack("<f", struct.pack("<f", v))[0]


def test_row_scale_equals_ieee_division_for_every_bf16():
    c = f32(Fraction(1, 127))
    assert float(c) == 0.007874015718698502      # kInv127 in titan_kv.cu
    floor = f32(Fraction(1, 10 ** 12))
    mismatches = []
    for bits in range(0x7F80):               # +0 .. largest finite bf16
        a = Fraction(struct.unpack("<f", struct.pack("<I", bits << 16))[0])
        want = max(f32(a / 127), floor)
        y0 = f32(a * c)
        y = f32(f32(a - y0 * 127) * c + y0)
        if max(y, floor) != want:
            mismatches.append(bits)
    assert not mismatches, mismatches[:10]
