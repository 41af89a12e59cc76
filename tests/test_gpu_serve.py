"""The decode server (ttl_moe_serve): blocking ttl_moe_decode calls answered
by a resident launch of the decode kernel through a mailbox in mapped pinned
memory.  Its answers equal the ordinary blocking call's bit for bit (same
kernel steps), also after the launch left for idleness and was started again,
and around other calls on the handle (which stop it first); and they match
tt-lab's CPU MoE (the oracle) within the parity bar."""
import time

import numpy as np
import pytest

import oracle
from conftest import synth_layer

pytestmark = pytest.mark.gpu

LAYERS = 3


@pytest.fixture(scope="module")
def handles():
    import ttl_moe
    layers = [synth_layer(60 + l, 32, layer=l) for l in range(LAYERS)]
    plain = ttl_moe.MoE(experts=32, layers=LAYERS, max_tokens=8, device=0)
    served = ttl_moe.MoE(experts=32, layers=LAYERS, max_tokens=8, device=0)
    for l, t in enumerate(layers):
        plain.upload_layer(l, t)
        served.upload_layer(l, t)
    served.serve(20000)  # leaves after 20 ms without a request
    yield plain, served, layers
    served.close()
    plain.close()


def same(a, b):
    return all(np.array_equal(x, y) for x, y in zip(a, b))


def test_served_decode_equals_plain_decode(handles):
    from ttl_moe import synth
    plain, served, layers = handles
    for k in range(12):
        x = synth.inputs_host(300 + k, 1)[0]
        l = k % LAYERS
        assert same(served.moe(l, x), plain.moe(l, x)), k
    x = synth.inputs_host(320, 1)[0]
    out, idx, w = served.moe(1, x)
    r_out, r_idx, r_w = oracle.moe_decode(layers[1], x, impl="ref" if oracle.ref_available() else "port")
    assert np.array_equal(idx, r_idx)
    assert oracle.compare(out, r_out)["max_rel"] <= 1e-3


def test_server_restarts_after_idle_and_around_other_calls(handles):
    from ttl_moe import synth
    plain, served, _ = handles
    x = synth.inputs_host(330, 1)[0]
    first = served.moe(0, x)
    time.sleep(0.1)  # the resident launch leaves (idle limit 20 ms)
    assert same(served.moe(0, x), first)
    xs = synth.inputs_host(331, 3)
    assert np.array_equal(served.forward(0, LAYERS, xs), plain.forward(0, LAYERS, xs))  # stops the server first
    assert same(served.moe(2, x), plain.moe(2, x))
    xb = synth.inputs_host(332, 5)
    assert np.array_equal(served.moe_batch(1, xb)[0], plain.moe_batch(1, xb)[0])
    assert same(served.moe(1, x), plain.moe(1, x))


def test_server_errors_and_off_switch(handles):
    import ttl_moe
    plain, served, _ = handles
    with pytest.raises(RuntimeError, match="out of range"):
        served.moe(LAYERS, np.zeros(2880, np.float32))
    with pytest.raises(RuntimeError, match="at most 1000000"):
        served.serve(2_000_000)
    from ttl_moe import synth
    x = synth.inputs_host(340, 1)[0]
    served.serve(0)
    assert same(served.moe(0, x), plain.moe(0, x))
    served.serve(20000)
    assert same(served.moe(0, x), plain.moe(0, x))
    with ttl_moe.MoE(experts=32, layers=2, device=0) as m:
        m.upload_layer(0, synth_layer(60, 32, layer=0))
        m.serve(20000)
        with pytest.raises(RuntimeError, match="every layer uploaded"):
            m.moe(0, x)
