"""The multi-token drivers of tt-lab's compiled CPU code (oracle/ref_shim.cpp)
that the full-size parity tests and bench.py's reference arm use: run on many
host threads, they must give exactly the single-threaded reference's results."""
import numpy as np
import pytest

import oracle
from oracle import synth as osynth

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def two_layers():
    return [osynth.layer_host(0, l, 32, norm=(l == 1)) for l in range(2)]


def test_forward_tokens_equals_sequential_reference(two_layers):
    x = osynth.inputs_host(0, 5)
    norms = [t.get("norm_w") for t in two_layers]
    y = oracle.forward_tokens(two_layers, x, threads=3, norms=norms)
    ref = oracle.forward(two_layers, x, impl="ref")
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


def test_layer_tokens_is_the_reference_moe(two_layers):
    t = two_layers[0]
    x = osynth.inputs_host(1, 4)
    y, idx, w, logits = oracle.moe_layer_tokens(t, x, threads=2)
    ones = np.ones(2880, np.float32)
    for i in range(4):
        h = oracle.rms_norm(x[i], ones, impl="ref")
        out, ridx, rw = oracle.moe_decode(t, h, impl="ref")
        assert np.array_equal(idx[i], ridx) and np.array_equal(w[i], rw)
        assert np.array_equal((x[i] + out).astype(np.float32).view(np.uint32), y[i].view(np.uint32))
        # the logits are tt-lab's router chain: bias first, products added in column order
        chain = t["router_b"].copy()
        for e in range(32):
            s = np.float32(t["router_b"][e])
            for c in range(0, 2880):
                s = np.float32(s + np.float32(t["router_w"][e * 2880 + c] * h[c]))
            chain[e] = s
            if e == 2:
                break
        assert np.array_equal(logits[i, :3], chain[:3])


def test_layer_major_equals_token_major(two_layers):
    x = osynth.inputs_host(2, 6)
    norms = [t.get("norm_w") for t in two_layers]
    h = x
    for t, g in zip(two_layers, norms):
        h, _, _, _ = oracle.moe_layer_tokens(t, h, norm_w=g, threads=4)
    y = oracle.forward_tokens(two_layers, x, threads=2, norms=norms)
    assert np.array_equal(h.view(np.uint32), y.view(np.uint32))
