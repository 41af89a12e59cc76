"""The GPU output head (ttl_head_*: rms_norm -> matvec_q8_0 -> greedy) against
the checker, bit for bit: logits and token equal tt-lab's (oracle/moe_oracle.c,
itself held to the compiled reference in tests/test_head_oracle.py)."""
import numpy as np
import pytest

import oracle
from oracle import synth as osynth

pytestmark = pytest.mark.gpu


def same_bits(a, b):
    nan = np.isnan(b)
    return np.array_equal(np.isnan(a), nan) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


def test_head_full_vocab_bit_exact():
    import ttl_moe
    V = oracle.VOCAB
    t = osynth.head_host(0, V)
    x = osynth.inputs_host(6, 3)
    with ttl_moe.Head(vocab=V, device=0) as h:
        h.upload(t["output_w"], t["output_norm"])
        for xi in x:
            logits, tok = h.forward(xi)
            rl, rt = oracle.head(t["output_w"], t["output_norm"], xi, V)
            assert same_bits(logits, rl)
            assert tok == rt == oracle.greedy(rl, "ref")
        # token only (no logits copy)
        _, tok = h.forward(x[0], want_logits=False)
        assert tok == oracle.head(t["output_w"], t["output_norm"], x[0], V)[1]


def test_head_hostile_scales_and_unpack():
    import ttl_moe
    from test_head_oracle import hostile_rows
    V = 320
    w = hostile_rows(V)
    g = osynth.normal_host(2880, 1, 9, 0.02, 1.0)
    x = osynth.inputs_host(7, 2)
    with ttl_moe.Head(vocab=V, device=0) as h:
        h.upload(w, g)
        assert np.array_equal(h.unpack(), w)
        for xi in x:
            logits, tok = h.forward(xi)
            rl, rt = oracle.head(w, g, xi, V)
            assert same_bits(logits, rl)
            assert tok == rt


def test_head_greedy_ties_and_nan():
    import ttl_moe
    V = 256
    base = osynth.q8_0_host(V * 90, 2, 5).reshape(V, 90, 34)
    g = np.ones(2880, np.float32)
    x = osynth.inputs_host(8, 1)[0]
    with ttl_moe.Head(vocab=V, device=0) as h:
        # rows 40 and 200 identical and the largest: the lower one wins
        w = base.copy()
        w[:, :, 2:] = 0
        w[40, :, 2:] = np.where(x.reshape(90, 32) > 0, 0x7F, 0x81).astype(np.uint8)
        w[200] = w[40]
        h.upload(np.ascontiguousarray(w.reshape(-1)), g)
        logits, tok = h.forward(x)
        assert tok == 40 == oracle.head(np.ascontiguousarray(w.reshape(-1)), g, x, V)[1]
        # a NaN logit at row 0 is never replaced (a NaN scale in row 0)
        w[0, 3, 0], w[0, 3, 1] = 0x00, 0x7E
        wb = np.ascontiguousarray(w.reshape(-1))
        h.upload(wb, g)
        logits, tok = h.forward(x)
        assert np.isnan(logits[0]) and tok == 0 == oracle.head(wb, g, x, V)[1]
