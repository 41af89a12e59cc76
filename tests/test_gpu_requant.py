"""requant --cuda end to end: a gpt-oss GGUF (two synthetic 20b layers) to a
TTQ file with GPU-layout experts (ttl_requant_gpu), read back by tt-lab's
own TtqFile (src/tt_backend.cpp:315-445), bound with
ttl_moe_upload_layer_packed and checked against the GGUF upload and tt-lab's
CPU MoE (the oracle).  Bar as in the parity tests: top-4 bit-exact, output
max error <= 1e-3 of max |reference|."""
import numpy as np
import pytest

import oracle
from gguf_write import gpt_oss_meta, moe_tensors, write_gguf

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.ttq_available(), reason="tt-lab TTQ reader not built")]

D = 2880
SEED = 11
LAYERS = (0, 1)
KINDS = ("gate", "up", "down")


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    from ttl_moe import synth
    d = tmp_path_factory.mktemp("requant")
    layers = {l: synth.layer_host(SEED, l, 32) for l in LAYERS}
    tensors = [x for l in LAYERS for x in moe_tensors(l, layers[l])]
    write_gguf(d / "m.gguf", gpt_oss_meta(), tensors)
    return d, layers


@pytest.fixture(scope="module")
def ttq(model):
    import ttl_moe
    d, _ = model
    ttl_moe.requant_gpu(d / "m.gguf", d / "m.ttq", 0, len(LAYERS), device=0)
    recs = oracle.ttq_read(d / "m.ttq")
    return recs, {r["name"]: r for r in recs}


def packed_layer(by_name, l):
    p = f"blk.{l}."
    f32 = lambda n: by_name[p + n]["payload"].view(np.float32)  # noqa: E731
    t = {"router_w": f32("ffn_gate_inp.weight"), "router_b": f32("ffn_gate_inp.bias")}
    for m in KINDS:
        t[f"{m}_p"] = by_name[p + f"ffn_{m}_exps.weight.mxfp4gpu"]["payload"]
        t[f"{m}_b"] = f32(f"ffn_{m}_exps.bias")
    return t


def test_ttq_records_as_tt_lab_reads_them(model, ttq):
    import ttl_moe
    _, layers = model
    recs, by_name = ttq
    assert recs.layers == 24 and len(recs) == 8 * len(LAYERS)
    expected = []
    for l in LAYERS:
        p = f"blk.{l}."
        expected += [(p + "ffn_gate_inp.weight", 7, [D, 32]), (p + "ffn_gate_inp.bias", 7, [32])]
        for m in KINDS:
            expected += [(p + f"ffn_{m}_exps.weight.mxfp4gpu", 6, [D, D, 32]), (p + f"ffn_{m}_exps.bias", 7, [D, 32])]
    assert [(r["name"], r["format"], r["shape"]) for r in recs] == expected
    for r in recs:
        assert r["payload"].ctypes.data % 64 == 0
    for l in LAYERS:
        p, t = f"blk.{l}.", layers[l]
        assert np.array_equal(by_name[p + "ffn_gate_inp.weight"]["payload"].view(np.float32), t["router_w"])
        assert np.array_equal(by_name[p + "ffn_gate_inp.bias"]["payload"].view(np.float32), t["router_b"])
        for m in KINDS:
            rec = by_name[p + f"ffn_{m}_exps.weight.mxfp4gpu"]["payload"]
            assert rec.nbytes == ttl_moe.packed_bytes(32)
            back = ttl_moe.unpack_mxfp4(rec, 32)  # lossless: the GGUF blocks come back exactly
            assert np.array_equal(back, t[f"{m}_w"]), (l, m)
            assert np.array_equal(by_name[p + f"ffn_{m}_exps.bias"]["payload"].view(np.float32), t[f"{m}_b"])


def test_requant_layer_subrange(model):
    import ttl_moe
    d, _ = model
    ttl_moe.requant_gpu(d / "m.gguf", d / "one.ttq", 1, 2, device=0)
    recs = oracle.ttq_read(d / "one.ttq")
    assert len(recs) == 8 and all(r["name"].startswith("blk.1.") for r in recs)


def test_packed_upload_matches_gguf_upload_and_reference(model, ttq):
    import ttl_moe
    from ttl_moe import synth
    _, layers = model
    _, by_name = ttq
    a = ttl_moe.MoE(experts=32, layers=len(LAYERS), max_tokens=64, device=0)
    b = ttl_moe.MoE(experts=32, layers=len(LAYERS), max_tokens=64, device=0)
    try:
        for l in LAYERS:
            a.upload_layer(l, layers[l])
            b.upload_layer_packed(l, packed_layer(by_name, l))
        for tok in range(3):
            x = synth.inputs_host(100 + tok, 1)[0]
            for l in LAYERS:
                ya, ia, wa = a.moe(l, x)
                yb, ib, wb = b.moe(l, x)
                assert np.array_equal(ya, yb) and np.array_equal(ia, ib) and np.array_equal(wa, wb)
                r_out, r_idx, r_w = oracle.moe_decode(layers[l], x, impl="ref" if oracle.ref_available() else "port")
                assert np.array_equal(ib, r_idx)
                np.testing.assert_allclose(wb, r_w, rtol=1e-5, atol=0)
                m = oracle.compare(yb, r_out)
                assert m["max_rel"] <= 1e-3, m
        x = synth.inputs_host(200, 48)
        assert np.array_equal(a.moe_batch(0, x)[0], b.moe_batch(0, x)[0])
        assert np.array_equal(a.forward(0, len(LAYERS), x), b.forward(0, len(LAYERS), x))
    finally:
        a.close()
        b.close()


def test_packed_upload_refuses_scale_255(ttq):
    import ttl_moe
    _, by_name = ttq
    t = packed_layer(by_name, 0)
    bad = t["down_p"].copy()
    bad[ttl_moe.packed_bytes(1) * 5 + D * D // 2 + 17] = 255  # a scale byte of expert 5
    t = dict(t, down_p=bad)
    m = ttl_moe.MoE(experts=32, layers=1, device=0)
    try:
        with pytest.raises(RuntimeError, match="scale byte is 255"):
            m.upload_layer_packed(0, t)
    finally:
        m.close()
