"""The attention restatement (oracle/attn_oracle.c) against tt-lab's own
attention block compiled from its sources (tref_attention_steps: rms_norm,
matvec_add_q8_0, the model's apply_rope / store_kv / attention_from_cache),
bit for bit, on a sliding-window layer past its window and on a full layer."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="reference not built")


@pytest.fixture(scope="module")
def attn_layer():
    from ttl_moe import synth
    return synth.attention_layer_host(5, 0)


@pytest.mark.parametrize("layer_index,positions", [(0, 136), (1, 24)])
def test_restatement_equals_reference(attn_layer, layer_index, positions):
    from ttl_moe import synth
    x = synth.inputs_host(70 + layer_index, positions)
    r_res, r_att = oracle.attention_steps(attn_layer, layer_index, x, impl="ref")
    p_res, p_att = oracle.attention_steps(attn_layer, layer_index, x, impl="port")
    assert np.isfinite(r_res).all()
    assert np.array_equal(p_att.view(np.uint32), r_att.view(np.uint32))
    assert np.array_equal(p_res.view(np.uint32), r_res.view(np.uint32))


def test_sliding_window_drops_old_positions(attn_layer):
    """Layer 0 (even) attends to the last 128 positions only: past the window
    its attention output no longer depends on position 0's value row, while
    layer 1's still does."""
    from ttl_moe import synth
    x = synth.inputs_host(80, 131)
    x2 = x.copy()
    x2[0] *= 3.0
    for layer_index, depends in ((0, False), (1, True)):
        a = oracle.attention_steps(attn_layer, layer_index, x, impl="port")[1]
        b = oracle.attention_steps(attn_layer, layer_index, x2, impl="port")[1]
        assert np.array_equal(a[130], b[130]) != depends
        assert not np.array_equal(a[5], b[5])
