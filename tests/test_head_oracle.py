"""The output head's checker (oracle/moe_oracle.c: matvec_q8_0, greedy, the
half conversion) held bit for bit to tt-lab's compiled code (oracle/_ref):
src/tensor.cpp:163-165, :202-218 and src/model.cpp:604-612."""
import numpy as np
import pytest

import oracle
from oracle import synth as osynth

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def hostile_rows(rows, seed=5):
    """Seeded Q8_0 rows with scales 0, subnormal, largest, inf, NaN and the
    int8 extremes mixed in."""
    w = osynth.q8_0_host(rows * 90, seed, 3).reshape(rows, 90, 34)
    specials = [0x0000, 0x0001, 0x03FF, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0x8000, 0x3C00]
    for r in range(rows):
        for k, h in enumerate(specials):
            if (r + k) % 5 == 0:
                b = (r * 7 + k * 11) % 90
                w[r, b, 0], w[r, b, 1] = h & 0xFF, h >> 8
    w[1, :, 2:] = 0x80   # -128 everywhere
    w[2, :, 2:] = 0x7F   # 127 everywhere
    return np.ascontiguousarray(w.reshape(-1))


def test_half_to_float_is_exact():
    h = np.arange(65536, dtype=np.uint16)
    f = np.array([oracle.port().oref_half_to_float(int(v)) for v in h], np.float32)
    g = h.view(np.float16).astype(np.float32)
    nan = np.isnan(g)
    assert np.array_equal(f.view(np.uint32)[~nan], g.view(np.uint32)[~nan])
    assert np.all(np.isnan(f[nan]))


@needs_ref
def test_matvec_q8_0_port_equals_reference():
    rows = 320
    x = osynth.inputs_host(0, 2)
    for w in (osynth.q8_0_host(rows * 90, 0, 11), hostile_rows(rows)):
        for xi in x:
            a = oracle.matvec_q8_0(w, xi, rows, "port")
            b = oracle.matvec_q8_0(w, xi, rows, "ref")
            nan = np.isnan(b)
            assert np.array_equal(np.isnan(a), nan)
            assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@needs_ref
def test_greedy_port_equals_reference():
    rng = np.random.default_rng(0)
    v = rng.standard_normal(oracle.VOCAB).astype(np.float32)
    cases = [v.copy() for _ in range(6)]
    cases[1][[10, 5000, 200000]] = 9.0          # a three-way tie: the first wins
    cases[2][0] = np.nan                         # NaN at 0 is never replaced
    cases[3][[7, 9]] = [np.nan, 50.0]            # NaNs elsewhere are passed over
    cases[4][:] = -0.0
    cases[4][3] = 0.0                            # -0 and +0 compare equal
    cases[5][:] = np.nan
    for c in cases:
        assert oracle.greedy(c, "port") == oracle.greedy(c, "ref")
