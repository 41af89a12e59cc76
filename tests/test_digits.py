"""The prefill B operand's digit encoding (tt-lab_b200/csrc/prefill_tc.cu),
restated in numpy and checked exhaustively on CPU.

A K-block value with magnitude m = |v| * 2^(16 - e) rounded to nearest (e the
exponent of the block's largest |v|, so 0 <= m <= 2^17) is
written as six balanced radix-8 digits c_d in [-4, 4], m = sum_d c_d 8^d,
each an exact E2M1 value with the sign of v applied, digit row d scaled by
2^(e - 16 + 3d).  radix8_codes computes the six E2M1 codes per nibble
without branches from the octal digits of m + 4 * (1 + 8 + ... + 8^4); these
tests hold that arithmetic to the digit-by-digit definition for every m and
both signs, and the reconstruction to m exactly.
"""
import numpy as np

E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6], np.float64)
ALL = np.arange((1 << 17) + 1, dtype=np.int64)  # every magnitude, 2^17 included


def digits_loop(m):
    """Balanced radix-8 digits by definition: c = ((r + 4) mod 8) - 4, carry the rest."""
    r = m.copy()
    out = []
    for _ in range(5):
        c = ((r + 4) & 7) - 4
        r = (r - c) >> 3
        out.append(c)
    out.append(r)
    return np.stack(out, axis=1)


def codes_swar(m, neg):
    """radix8_codes (prefill_tc.cu), word for word in numpy."""
    m = m.astype(np.uint64)
    mp = m + 0x4924
    o = ((mp & 0x7) | ((mp << 1) & 0x70) | ((mp << 2) & 0x700) | ((mp << 3) & 0x7000) | ((mp << 4) & 0x70000)
         | ((mp << 5) & 0x700000))
    up = (o >> 2) & 0x11111
    up_mask = up * 0xF
    a_up = o & 0x33333
    a_down = ((~o) & 0x33333) + 0x11111
    a = (a_up & up_mask) | (a_down & ~up_mask & 0xFFFFF) | (o & 0xF00000)
    big = ((a + 0x111111) >> 2) & 0x111111
    big_mask = big * 0xF
    code = ((a << 1) & ~big_mask) | ((a + 0x222222) & big_mask)
    nonzero = (a | (a >> 1) | (a >> 2)) & 0x111111
    negmask = np.uint64(0x111111) if neg else np.uint64(0)
    sign = ((~up & 0x11111) ^ negmask) & nonzero
    return (code | (sign << 3)) & 0xFFFFFFFF


def test_digits_are_balanced_and_exact():
    c = digits_loop(ALL)
    assert c[:, :5].min() >= -4 and c[:, :5].max() <= 3
    assert c[:, 5].min() >= 0 and c[:, 5].max() <= 4
    assert np.array_equal((c * (8 ** np.arange(6))).sum(axis=1), ALL)


def test_swar_codes_match_the_digit_definition():
    c = digits_loop(ALL)
    mag = np.abs(c)
    code_of = np.array([0, 2, 4, 5, 6], np.uint64)  # E2M1 codes of 0, 1, 2, 3, 4
    for neg in (0, 1):
        want = np.zeros(ALL.size, np.uint64)
        for d in range(6):
            sign = ((c[:, d] < 0).astype(np.uint64) ^ np.uint64(neg)) & (c[:, d] != 0).astype(np.uint64)
            want |= (code_of[mag[:, d]] | (sign << np.uint64(3))) << np.uint64(4 * d)
        assert np.array_equal(codes_swar(ALL, neg), want)


def test_codes_reconstruct_the_magnitude():
    for neg in (0, 1):
        codes = codes_swar(ALL, neg)
        total = np.zeros(ALL.size, np.float64)
        for d in range(6):
            nib = (codes >> np.uint64(4 * d)) & np.uint64(0xF)
            val = E2M1[(nib & np.uint64(7)).astype(np.int64)] * np.where(nib & np.uint64(8), -1.0, 1.0)
            total += val * 8.0 ** d
        assert np.array_equal(total, (-1.0 if neg else 1.0) * ALL.astype(np.float64))
        assert not np.any((codes >> np.uint64(24)) & np.uint64(0xFF))  # nibbles 6, 7 stay zero


def test_digit_scales():
    """digit_scales6: E8M0 of 2^(e - 16 + 3d) is code - (16 - 3d), saturating at 0,
    and the NaN code 255 stays 255."""
    codes = np.arange(256)
    for d in range(6):
        got = np.where(codes == 255, 255, np.maximum(codes - (16 - 3 * d), 0))
        # the packed form of the kernel: byte-wise saturating subtract, NaN bytes kept
        packed = np.array([max(int(c) - (16 - 3 * d), 0) if c != 255 else 255 for c in codes])
        assert np.array_equal(got, packed)
        # a normal block (code = e + 127) gives row d the scale 2^(e - 16 + 3d)
        e = np.arange(-100, 100)
        assert np.array_equal(np.maximum(e + 127 - (16 - 3 * d), 0) - 127, e - 16 + 3 * d)


def test_rounded_magnitudes_stay_within_the_digits_and_half_a_step():
    """m = rint(|v| 2^(16-e)) for the block maximum's exponent e: m <= 2^17
    (what six balanced digits hold), and |v - m 2^(e-16)| <= 2^(e-17)."""
    rng = np.random.default_rng(5)
    v = rng.standard_normal((4096, 32)).astype(np.float32) * np.float32(2.0) ** rng.integers(-60, 60, (4096, 1))
    v[0, :] = np.nextafter(np.float32(2.0), np.float32(0))  # the largest value below a power of two rounds up to 2^17
    mb = np.abs(v).max(axis=1, keepdims=True)
    e = np.floor(np.log2(mb.astype(np.float64)))
    m = np.rint(np.abs(v).astype(np.float64) * 2.0 ** (16 - e))
    assert m.max() == 1 << 17
    c = digits_loop(m.astype(np.int64).ravel())
    assert c[:, 5].max() <= 4
    assert np.all(np.abs(np.abs(v) - m * 2.0 ** (e - 16)) <= 2.0 ** (e - 17))
