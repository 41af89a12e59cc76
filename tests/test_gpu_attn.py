"""The attention block on the GPU (ttl_attn_*) against tt-lab's own
attention code (the oracle: tref_attention_steps, or the bit-exact C
restatement): rms_norm, Q / K / V Q8_0 projections, YaRN RoPE, the KV cache,
attention with sinks (even layers: sliding window of 128), the output
projection and the residual, position by position.

Bar: max |gpu - ref| <= 1e-3 of max |ref| per position (the parity tests'
bar; the GPU's RMS norm is a tree sum and its cos / sin / exp are CUDA's, so
the results are not bit-identical)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-3


def impl():
    return "ref" if oracle.ref_available() else "port"


def rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b)))


@pytest.fixture(scope="module")
def layers():
    from ttl_moe import synth
    return [synth.attention_layer_host(5, l) for l in range(2)]


def test_attention_matches_reference_position_by_position(layers):
    import ttl_moe
    from ttl_moe import synth
    runs = ((0, 140), (1, 40))  # a sliding layer past its window, a full layer
    with ttl_moe.Attention(layers=2, token_capacity=160, device=0) as a:
        for l, t in enumerate(layers):
            a.upload_layer(l, t)
        for l, P in runs:
            x = synth.inputs_host(90 + l, P)
            r_res, r_att = oracle.attention_steps(layers[l], l, x, impl=impl())
            worst_res = worst_att = 0.0
            for p in range(P):
                res, att = a.forward(l, p, x[p])
                worst_res = max(worst_res, rel(res, r_res[p]))
                worst_att = max(worst_att, rel(att, r_att[p]))
            assert worst_att <= TOL, (l, worst_att)
            assert worst_res <= TOL, (l, worst_res)


def test_attention_long_context_tiles(layers):
    """A full-attention layer to 1040 positions: each of the 8 splits of the
    window then spans three staged tiles of 64 positions (the third refills
    the first buffer), checked at every position."""
    import ttl_moe
    from ttl_moe import synth
    P = 1040
    x = synth.inputs_host(91, P)
    r_res, r_att = oracle.attention_steps(layers[1], 1, x, impl=impl())
    with ttl_moe.Attention(layers=2, token_capacity=P, device=0) as a:
        a.upload_layer(1, layers[1])
        worst_res = worst_att = 0.0
        for p in range(P):
            res, att = a.forward(1, p, x[p])
            worst_res = max(worst_res, rel(res, r_res[p]))
            worst_att = max(worst_att, rel(att, r_att[p]))
    assert worst_att <= TOL, worst_att
    assert worst_res <= TOL, worst_res


def test_attention_errors_follow_reference(layers):
    import ttl_moe
    x = np.zeros(2880, np.float32)
    with ttl_moe.Attention(layers=2, token_capacity=4, device=0) as a:
        with pytest.raises(RuntimeError, match="was not uploaded"):
            a.forward(0, 0, x)
        a.upload_layer(0, layers[0])
        with pytest.raises(RuntimeError, match="position exceeds startup token capacity"):
            a.forward(0, 4, x)
        with pytest.raises(RuntimeError, match="out of range"):
            a.forward(2, 0, x)
        res, _ = a.forward(0, 0, x)  # the handle stays usable
        assert np.isfinite(res).all()


def test_gpu_resident_decode_layer(layers):
    """Attention and the MoE half of a layer chained on one stream in device
    memory (no host round trip inside the layer), for a few positions, against
    the oracle's attention block followed by its rms_norm -> moe -> residual."""
    import torch
    import ttl_moe
    from conftest import synth_layer
    from ttl_moe import synth
    moe_t = synth_layer(21, 32, layer=0, norm=True)
    P = 6
    x = synth.inputs_host(95, P)
    with ttl_moe.MoE(experts=32, layers=1, device=0) as m, \
            ttl_moe.Attention(layers=1, token_capacity=P, device=0, stream=m.stream()) as a:
        m.upload_layer(0, moe_t)
        a.upload_layer(0, layers[0])
        xd = torch.from_numpy(x).cuda()
        rd = torch.empty_like(xd)
        yd = torch.empty_like(xd)
        for p in range(P):
            a.forward_async(0, p, xd[p], rd[p])
            m.forward_async(0, 1, rd[p], yd[p], 1)
        m.sync()
        y = yd.cpu().numpy()
    r_res, _ = oracle.attention_steps(layers[0], 0, x, impl=impl())
    r_y = oracle.forward([moe_t], r_res, impl=impl())
    for p in range(P):
        assert rel(y[p], r_y[p]) <= TOL, p
