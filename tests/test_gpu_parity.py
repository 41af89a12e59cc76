"""GPU parity of the CUDA MoE path against tt-lab's CPU MoE (the oracle).

Bar: top-4 indices bit-exact (no near-tie
exemption is needed: the decode router re-evaluates near-ties in the
reference's own order, the prefill router always uses it); MoE output max
error <= 1e-3 relative to max |reference output|, f32 accumulation.
All calls go through the C ABI (libttl_moe) with host buffers.
"""
import numpy as np
import pytest

import oracle
from conftest import synth_layer

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max |gpu - ref| / max |ref|
D = 2880


def impl():
    return "ref" if oracle.ref_available() else "port"


@pytest.fixture(scope="module")
def ttl():
    import ttl_moe
    ttl_moe.lib()
    return ttl_moe


@pytest.fixture(scope="module")
def moe32(ttl, layer32):
    m = ttl.MoE(experts=32, layers=2, max_tokens=512, device=0)
    m.upload_layer(0, layer32)
    yield m
    m.close()


@pytest.fixture(scope="module")
def moe128(ttl, layer128):
    m = ttl.MoE(experts=128, layers=1, max_tokens=64, device=0)
    m.upload_layer(0, layer128)
    yield m
    m.close()


def assert_close(out, ref, tol=TOL):
    m = oracle.compare(out, ref)
    assert m["max_rel"] <= tol, m
    return m


@pytest.mark.parametrize("token", range(4))
def test_decode_20b_matches_reference(moe32, layer32, token):
    from ttl_moe import synth
    x = synth.inputs_host(token, 1)[0]
    out, idx, w = moe32.moe(0, x)
    r_out, r_idx, r_w = oracle.moe_decode(layer32, x, impl=impl())
    assert np.array_equal(idx, r_idx)
    np.testing.assert_allclose(w, r_w, rtol=1e-5, atol=0)
    assert_close(out, r_out)


@pytest.mark.parametrize("token", range(2))
def test_decode_120b_matches_reference(moe128, layer128, token):
    from ttl_moe import synth
    x = synth.inputs_host(50 + token, 1)[0]
    out, idx, w = moe128.moe(0, x)
    r_out, r_idx, r_w = oracle.moe_decode(layer128, x, impl=impl())
    assert np.array_equal(idx, r_idx)
    np.testing.assert_allclose(w, r_w, rtol=1e-5, atol=0)
    assert_close(out, r_out)


def test_decode_exact_ties_follow_reference_order(ttl):
    """Router rows engineered to tie exactly: the GPU must reproduce the
    reference selection sort's tie order (src/model.cpp:296-309)."""
    from test_oracle import tie_layer
    t = tie_layer()
    with ttl.MoE(experts=32, layers=1, device=0) as m:
        m.upload_layer(0, t)
        x = np.zeros(D, np.float32)
        x[::7] = 0.5
        out, idx, w = m.moe(0, x)
        r_out, r_idx, r_w = oracle.moe_decode(t, x, impl=impl())
        assert np.array_equal(idx, r_idx), (idx, r_idx)
        assert m.counters()["router_exact_reevals"] >= 1
        assert_close(out, r_out)


def test_prefill_exact_ties_follow_reference_order(ttl):
    """The prefill router's parallel ranking must hand exact ties to the
    selection sort (src/model.cpp:344-357): tokens whose logits tie at the top,
    mixed with tokens without ties."""
    from test_oracle import tie_layer
    from ttl_moe import synth
    t = tie_layer()
    x = synth.inputs_host(5, 6)
    x[0] = 0.0
    x[0, ::7] = 0.5
    x[1] = 0.0
    x[2] = 0.0
    x[2, 1::5] = -0.25
    x[4] = x[0]
    with ttl.MoE(experts=32, layers=1, max_tokens=8, device=0) as m:
        m.upload_layer(0, t)
        out, idx, w = m.moe_batch(0, x)
    r_out, r_idx, r_w = oracle.moe_prefill(t, x, impl=impl())
    assert len({3, 9, 17} & set(r_idx[1])) >= 2
    assert np.array_equal(idx, r_idx), (idx, r_idx)
    np.testing.assert_allclose(w, r_w, rtol=1e-5, atol=0)
    assert_close(out, r_out)


@pytest.mark.parametrize("tokens", [1, 3, 17, 64])
def test_prefill_matches_reference(moe32, layer32, tokens):
    from ttl_moe import synth
    x = synth.inputs_host(1000 + tokens, tokens)
    out, idx, w = moe32.moe_batch(0, x)
    r_out, r_idx, r_w = oracle.moe_prefill(layer32, x, impl=impl())
    assert np.array_equal(idx, r_idx)
    np.testing.assert_allclose(w, r_w, rtol=1e-5, atol=0)
    assert_close(out, r_out)


def test_prefill_120b_matches_reference(moe128, layer128):
    from ttl_moe import synth
    x = synth.inputs_host(77, 40)
    out, idx, w = moe128.moe_batch(0, x)
    r_out, r_idx, r_w = oracle.moe_prefill(layer128, x, impl=impl())
    assert np.array_equal(idx, r_idx)
    assert_close(out, r_out)


def test_prefill_zipf_512_matches_reference(ttl):
    """Config 2: T = 512, router bias Zipf(1.1)-skewed (some experts get many
    tokens, some none)."""
    from ttl_moe import synth
    t = synth_layer(2, 32, zipf_s=1.1)
    x = synth.inputs_host(2, 512)
    with ttl.MoE(experts=32, layers=1, max_tokens=512, device=0) as m:
        m.upload_layer(0, t)
        out, idx, w = m.moe_batch(0, x)
    r_out, r_idx, r_w = oracle.moe_prefill(t, x, impl=impl())
    counts = np.bincount(r_idx.ravel(), minlength=32)
    assert counts.max() >= 3 * counts.mean()
    assert np.array_equal(idx, r_idx)
    assert_close(out, r_out)


def test_forward_stack_matches_reference(ttl):
    """RMSNorm -> MoE -> residual over 2 layers for 3 tokens (config 1 per-token step)."""
    from ttl_moe import synth
    layers = [synth_layer(10 + l, 32, layer=l, norm=True) for l in range(2)]
    x = synth.inputs_host(9, 3)
    with ttl.MoE(experts=32, layers=2, device=0) as m:
        for l, t in enumerate(layers):
            m.upload_layer(l, t)
        y = m.forward(0, 2, x)
    r = oracle.forward(layers, x, impl=impl())
    # per token, relative to the residual stream's magnitude
    for k in range(3):
        assert_close(y[k], r[k])


def test_forward_stack_120b_matches_reference(ttl):
    """gpt-oss-120b shapes (128 experts): RMSNorm -> MoE -> residual over 2
    layers for 2 tokens; the down reducers stage the next layer's router
    weights past the first 32 experts through shared memory."""
    from ttl_moe import synth
    layers = [synth_layer(70 + l, 128, layer=l, norm=True) for l in range(2)]
    x = synth.inputs_host(71, 2)
    with ttl.MoE(experts=128, layers=2, device=0) as m:
        for l, t in enumerate(layers):
            m.upload_layer(l, t)
        y = m.forward(0, 2, x)
    r = oracle.forward(layers, x, impl=impl())
    for k in range(2):
        assert_close(y[k], r[k])


def test_forward_graph_replay_with_new_inputs(ttl):
    """The second forward call on the same buffers replays the captured graph;
    with new inputs its outputs must follow them (the split-K partials carry
    per-launch tags, so a replay never reads the previous launch's words)."""
    from ttl_moe import synth
    layers = [synth_layer(20 + l, 32, layer=l, norm=True) for l in range(2)]
    xa = synth.inputs_host(31, 4)
    xb = synth.inputs_host(32, 4)
    with ttl.MoE(experts=32, layers=2, device=0) as m:
        for l, t in enumerate(layers):
            m.upload_layer(l, t)
        m.forward(0, 2, xa)
        yb = m.forward(0, 2, xb)
        ya = m.forward(0, 2, xa)
    rb = oracle.forward(layers, xb, impl=impl())
    ra = oracle.forward(layers, xa, impl=impl())
    for k in range(4):
        assert_close(yb[k], rb[k])
        assert_close(ya[k], ra[k])


def test_pack_roundtrip_hostile_bytes(ttl):
    rng = np.random.default_rng(3)
    g = rng.integers(0, 256, 2 * ttl.GGUF_MATRIX_BYTES, dtype=np.uint8)
    g.reshape(-1, 17)[:, 0] = rng.choice(np.array([0, 1, 2, 6, 7, 127, 253, 254, 255], np.uint8),
                                         g.size // 17)
    packed = ttl.pack_mxfp4(g, 2)
    assert packed.nbytes == ttl.packed_bytes(2)
    back = ttl.unpack_mxfp4(packed, 2)
    assert np.array_equal(back, g)
    # nibble order: element 2j in the low nibble of byte j; scales split out
    blk = g[:17]
    row0 = packed[:16]
    elems = np.concatenate([blk[1:17] & 15, blk[1:17] >> 4])
    assert np.array_equal(row0 & 15, elems[0::2]) and np.array_equal(row0 >> 4, elems[1::2])
    assert packed[2880 * 1440] == blk[0]


def test_errors_match_reference_behaviour(ttl, layer32):
    with ttl.MoE(experts=32, layers=2, max_tokens=4, device=0) as m:
        m.upload_layer(0, layer32)
        with pytest.raises(RuntimeError, match="not uploaded"):
            m.moe(1, np.zeros(D, np.float32))
        with pytest.raises(RuntimeError, match="startup batch capacity"):
            m.moe_batch(0, np.zeros((5, D), np.float32))
        with pytest.raises(RuntimeError, match="out of range"):
            m.moe(2, np.zeros(D, np.float32))
        out, idx, w = m.moe(0, np.zeros(D, np.float32))  # handle still usable
        assert np.isfinite(out).all()


def test_scale_byte_255_is_rejected_at_upload(ttl, layer32):
    """tt-lab reads E8M0 byte 255 as 2^128 (src/tensor.cpp:36-44); the tensor
    cores' E8M0 255 is NaN, so the upload refuses such weights loudly."""
    t = dict(layer32)
    bad = layer32["down_w"].copy()
    bad[17 * 1000] = 255  # the scale byte of one block
    t["down_w"] = bad
    with ttl.MoE(experts=32, layers=1, device=0) as m:
        with pytest.raises(RuntimeError, match="scale byte is 255"):
            m.upload_layer(0, t)
        m.upload_layer(0, layer32)  # the handle stays usable
        out, idx, w = m.moe(0, np.zeros(D, np.float32))
        assert np.isfinite(out).all()
