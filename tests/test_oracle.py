"""Pins the CPU oracle (tests only run it as the checker).

1. The reference's own known-answer vectors (tt-lab tests/host_dispatch.cpp:92-127,
   src/tests.cpp:42) on the C restatement and on the compiled reference.
2. Bit-exact agreement of the restatement with tt-lab's own GptOssModel::moe /
   moe_batch compiled from its sources (oracle/_ref), on seeded layers,
   hostile E8M0 scales and exact router ties.
"""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import synth_layer

D = 2880
BLOCKS = 90
EXPERT_BYTES = D * BLOCKS * 17

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def isa_here():
    if oracle.ref_available() and oracle.ref().tref_isa_v4():
        return oracle.ISA_V4
    return oracle.ISA_DEFAULT


def known_answer_weights():
    """Two experts; expert 1 has scale byte 127 and quant bytes 0x21 (tests/host_dispatch.cpp:95-101)."""
    data = np.zeros(2 * EXPERT_BYTES, np.uint8)
    blocks = data[EXPERT_BYTES:].reshape(-1, 17)
    blocks[:, 0] = 127
    blocks[:, 1:] = 0x21
    biases = np.full(2 * D, 0.25, np.float32)
    return data, biases


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_e8m0_scale_pins():
    # src/tests.cpp:42: mxfp4_scale(127) == 0.5; the table is 2^(e-128) for every byte.
    assert oracle.port().oref_mxfp4_scale(127) == 0.5
    for e in range(256):
        expect = np.float32(np.ldexp(1.0, e - 128))
        assert np.float32(oracle.port().oref_mxfp4_scale(e)) == expect
        if oracle.ref_available():
            assert np.float32(oracle.ref().tref_mxfp4_scale(e)) == expect


@pytest.mark.parametrize("isa", [oracle.ISA_DEFAULT, oracle.ISA_V4])
def test_known_answer_matvec_port(isa):
    data, biases = known_answer_weights()
    x = np.full(D, 0.5, np.float32)
    y = np.empty(D, np.float32)
    oracle.port().oref_matvec_add_mxfp4(data[EXPERT_BYTES:].ctypes.data, biases[D:].ctypes.data, x.ctypes.data,
                                        y.ctypes.data, isa)
    assert np.all(y == np.float32(1080.25))


@needs_ref
@pytest.mark.parametrize("isa", [-1, 0, 1])
def test_known_answer_matvec_reference(isa):
    if isa == 1 and not oracle.ref().tref_isa_v4():
        pytest.skip("host lacks x86-64-v4")
    data, biases = known_answer_weights()
    x = np.full(D, 0.5, np.float32)
    y = np.empty(D, np.float32)
    assert oracle.ref().tref_matvec_add_mxfp4(data.ctypes.data, biases.ctypes.data, 2, 1, x.ctypes.data,
                                              y.ctypes.data, isa) == 0
    assert np.all(y == np.float32(1080.25))


@pytest.mark.parametrize("count", [3, 16, 17])
@pytest.mark.parametrize("isa", [oracle.ISA_DEFAULT, oracle.ISA_V4])
def test_known_answer_matmul(count, isa):
    # tests/host_dispatch.cpp:108-126: token s (stored at slot count-s) sees input
    # (s+1)/2 and must give 1080*(s+1) + 0.25; the unselected token 0 stays -1.
    data, biases = known_answer_weights()
    tokens = np.array([count - s for s in range(count)], np.uint64)
    xt = np.empty(D * count, np.float32)
    for s in range(count):
        xt[s::count] = (s + 1) * 0.5
    impls = [("port", isa)]
    if oracle.ref_available() and (isa == 0 or oracle.ref().tref_isa_v4()):
        impls.append(("ref", isa))
    for impl, which in impls:
        out = np.full((count + 1) * D, -1.0, np.float32)
        if impl == "port":
            oracle.port().oref_matmul_add_mxfp4_selected(data[EXPERT_BYTES:].ctypes.data, biases[D:].ctypes.data,
                                                         xt.ctypes.data, tokens.ctypes.data, count, out.ctypes.data,
                                                         which)
        else:
            assert oracle.ref().tref_matmul_add_mxfp4_selected(data.ctypes.data, biases.ctypes.data, 2, 1,
                                                               xt.ctypes.data, tokens.ctypes.data, count,
                                                               out.ctypes.data, which) == 0
        o = out.reshape(count + 1, D)
        assert np.all(o[0] == -1.0), impl
        for s in range(count):
            assert np.all(o[tokens[s]] == np.float32(1080.0 * (s + 1) + 0.25)), (impl, s)


@needs_ref
@pytest.mark.parametrize("seed,experts", [(0, 32), (3, 32), (1, 128)])
def test_port_equals_reference_decode(seed, experts):
    from ttl_moe import synth
    t = synth_layer(seed, experts)
    for k in range(2):
        x = synth.inputs_host(seed + 100 * k, 1)[0]
        a = oracle.moe_decode(t, x, isa_here(), "port")
        b = oracle.moe_decode(t, x, impl="ref")
        assert np.array_equal(a[1], b[1])
        assert np.array_equal(bits(a[2]), bits(b[2]))
        assert np.array_equal(bits(a[0]), bits(b[0]))


@needs_ref
@pytest.mark.parametrize("tokens", [1, 6, 24])
def test_port_equals_reference_prefill(tokens):
    from ttl_moe import synth
    t = synth_layer(0, 32)
    x = synth.inputs_host(7, tokens)
    a = oracle.moe_prefill(t, x, isa_here(), "port")
    b = oracle.moe_prefill(t, x, impl="ref")
    assert np.array_equal(a[1], b[1])
    assert np.array_equal(bits(a[2]), bits(b[2]))
    assert np.array_equal(bits(a[0]), bits(b[0]))
    counts = np.bincount(b[1].ravel(), minlength=32)
    if tokens == 24:
        # both the <= 4-token matvec path and the gathered matmul path ran
        assert counts.max() > 4 and 0 < counts[counts > 0].min() <= 4


@needs_ref
@pytest.mark.parametrize("clone", [0, 1])
def test_hostile_scales_bit_exact(clone):
    # src/tests.cpp:168 uses scale bytes {0,1,2,6,7,127,253,254,255}.
    if clone == 1 and not oracle.ref().tref_isa_v4():
        pytest.skip("host lacks x86-64-v4")
    rng = np.random.default_rng(5)
    data = rng.integers(0, 256, EXPERT_BYTES, dtype=np.uint8)
    blocks = data.reshape(-1, 17)
    hostile = np.array([0, 1, 2, 6, 7, 127, 253, 254, 255], np.uint8)
    blocks[:, 0] = hostile[rng.integers(0, hostile.size, blocks.shape[0])]
    bias = rng.standard_normal(D).astype(np.float32)
    x = rng.standard_normal(D).astype(np.float32)
    y_port = np.empty(D, np.float32)
    y_ref = np.empty(D, np.float32)
    oracle.port().oref_matvec_add_mxfp4(data.ctypes.data, bias.ctypes.data, x.ctypes.data, y_port.ctypes.data, clone)
    assert oracle.ref().tref_matvec_add_mxfp4(data.ctypes.data, bias.ctypes.data, 1, 0, x.ctypes.data,
                                              y_ref.ctypes.data, clone) == 0
    assert np.array_equal(y_port, y_ref, equal_nan=True)


def tie_layer(experts=32):
    """A layer whose router has exact ties: experts 3, 9 and 17 share one row and
    bias; experts 5 and 30 share another (so the selection sort's tie rule decides)."""
    t = dict(synth_layer(0, experts))
    rw = t["router_w"].reshape(experts, D).copy()
    rb = t["router_b"].copy()
    rw[[9, 17]] = rw[3]
    rb[[9, 17]] = rb[3] = 0.6
    rw[30] = rw[5]
    rb[30] = rb[5] = 0.55
    rw[[3, 9, 17, 5, 30]] *= 0.01  # bias decides: ties at the top
    t["router_w"] = rw.reshape(-1)
    t["router_b"] = rb
    return t


@needs_ref
def test_tie_order_matches_reference():
    t = tie_layer()
    x = np.zeros(D, np.float32)
    x[::7] = 0.5
    a = oracle.moe_decode(t, x, isa_here(), "port")
    b = oracle.moe_decode(t, x, impl="ref")
    assert list(b[1][:3]) == [3, 9, 17] or len(set(b[1]) & {3, 9, 17}) >= 3
    assert np.array_equal(a[1], b[1])
    assert np.array_equal(bits(a[0]), bits(b[0]))


def test_select_top4_tie_rule():
    # Values [5, 7, 7, 1, 7]: pass 0 picks position 1 (first 7) and swaps it to
    # the front, leaving order [1, 0, 2, 3, 4]; pass 1 picks expert 2, pass 2
    # expert 4; then 0 (value 5).
    vals = np.array([5, 7, 7, 1, 7], np.float32)
    idx = np.empty(4, np.int32)
    oracle.port().oref_select_top4(vals.ctypes.data, 5, idx.ctypes.data)
    assert list(idx) == [1, 2, 4, 0]
    # A case where the swap makes the tie rule differ from "lowest index":
    # [5, 1, 5, 9]: pass 0 moves expert 3 to the front and expert 0 to the back
    # (order [3, 1, 2, 0]); pass 1 then meets expert 2 before expert 0, so the
    # tie between them goes to the higher id.
    vals = np.array([5, 1, 5, 9], np.float32)
    oracle.port().oref_select_top4(vals.ctypes.data, 4, idx.ctypes.data)
    assert list(idx) == [3, 2, 0, 1]


def test_swiglu_clamps():
    f = oracle.port().oref_swiglu
    assert f(100.0, 0.0) == pytest.approx(7.0 / (1.0 + np.exp(-1.702 * 7.0)), rel=1e-7)
    assert f(-100.0, 0.0) == pytest.approx(-100.0 / (1.0 + np.exp(170.2)), abs=1e-30)  # gate not clamped below
    assert f(1.0, 100.0) == pytest.approx(8.0 / (1.0 + np.exp(-1.702)), rel=1e-7)
    assert f(1.0, -100.0) == pytest.approx(-6.0 / (1.0 + np.exp(-1.702)), rel=1e-7)
