"""CPU checks of the integer / fp64 identities the dropout keep-mask kernel relies on
(flash-attention-rdna2_b200/csrc/dropout.cu):

* the high half of a 32 x 32 -> 64-bit Philox product from one round-down fused multiply-add,
  fma_rd(M * 2^-32, 2^52 + x, 2^52 - M * 2^20) = 2^52 + floor(M x / 2^32): both double constants
  are exact, the exact sum lies in [2^52, 2^53) (where doubles are the integers, so rounding down
  is the floor), and the low 32 bits of the result are (M x) >> 32;
* the keep test of the reference (kernels/fa_common.hpp:71-88), u = (r0 >> 8) / 2^24 >= p, as
  r0 >= ceil(p 2^24) << 8.
The GPU tests compare the kernel's bits with the oracle's Philox; these pin the arithmetic itself.
"""
import math
import struct
from fractions import Fraction

import numpy as np

PHILOX_M = (0xD2511F53, 0xCD9E8D57)


def _fma_rd_exact(a, b, c):
    """Exact a*b + c of doubles, rounded down to a double (exact rationals)."""
    v = Fraction(a) * Fraction(b) + Fraction(c)
    f = math.floor(v)
    assert 2 ** 52 <= f < 2 ** 53          # doubles in this binade are the integers
    return float(f)


def _low_word(d):
    return struct.unpack("<Q", struct.pack("<d", d))[0] & 0xFFFFFFFF


def _hilo_double(hi, lo):
    return struct.unpack("<d", struct.pack("<Q", (hi << 32) | lo))[0]


def test_fp64_high_half_constants_are_exact():
    for m in PHILOX_M:
        scaled = float(m) * 2.0 ** -32
        bias = 2.0 ** 52 - float(m) * 2.0 ** 20
        assert Fraction(scaled) == Fraction(m, 2 ** 32)
        assert Fraction(bias) == 2 ** 52 - m * 2 ** 20


def test_fp64_high_half_matches_integer_product():
    rng = np.random.default_rng(0)
    xs = [0, 1, 2, 0x7FFFFFFF, 0x80000000, 0xFFFFFFFE, 0xFFFFFFFF] + [int(v) for v in rng.integers(0, 2 ** 32, 2000)]
    for m in PHILOX_M:
        scaled, bias = float(m) * 2.0 ** -32, 2.0 ** 52 - float(m) * 2.0 ** 20
        for x in xs:
            xd = _hilo_double(0x43300000, x)
            assert xd == 2.0 ** 52 + x
            got = _low_word(_fma_rd_exact(scaled, xd, bias))
            assert got == (m * x) >> 32, (hex(m), x)


def test_keep_threshold_on_raw_word():
    rng = np.random.default_rng(1)
    rs = [0, 255, 256, 0xFFFFFF00, 0xFFFFFFFF] + [int(v) for v in rng.integers(0, 2 ** 32, 4000)]
    for p in (np.float32(1e-7), np.float32(0.1), np.float32(0.5), np.float32(0.3), np.nextafter(np.float32(1), 0)):
        thresh = math.ceil(float(p) * 2 ** 24)          # fa_drop_thresh
        assert thresh < 2 ** 24                         # thresh << 8 fits in 32 bits for p < 1
        for r in rs:
            keep_ref = (r >> 8) * (1.0 / 16777216.0) >= float(p)
            assert (r >= (thresh << 8)) == keep_ref == ((r >> 8) >= thresh)
