"""Golden fixtures of the MoE path (tests/golden/*.npz, written by
tests/golden/make_golden.py from tt-lab's own compiled CPU code).

CPU: the oracle's C restatement reproduces every fixture bit for bit with the
same instruction-set clone the reference ran -- this pins the oracle without
the reference sources (they are absent on the GPU box).
GPU: the CUDA path reproduces the fixtures' top-4 indices exactly and their
outputs within the north star's tolerance (max error <= 1e-3 of max |ref|).
"""
import json
import pathlib

import numpy as np
import pytest

import oracle
from conftest import synth_layer

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "golden.json").read_text())
ISA = oracle.ISA_V4 if META["reference_clone"] == "x86-64-v4" else oracle.ISA_DEFAULT
TOL = 1e-3


def load(name):
    return dict(np.load(GOLDEN / name))


def decode_layer():
    spec = META["fixtures"]["decode_e32.npz"]["layer"]
    return synth_layer(spec["seed"], spec["experts"], layer=spec["layer"])


def forward_layers():
    return [synth_layer(s["seed"], s["experts"], layer=s["layer"], norm=s["norm"])
            for s in META["fixtures"]["forward_e32_l2.npz"]["layers"]]


def test_fixture_files_are_described():
    for name in META["fixtures"]:
        assert (GOLDEN / name).exists(), name


def test_port_reproduces_decode_fixture():
    g = load("decode_e32.npz")
    t = decode_layer()
    for k in range(g["x"].shape[0]):
        y, idx, w = oracle.moe_decode(t, g["x"][k], isa=ISA, impl="port")
        assert np.array_equal(idx, g["idx"][k])
        assert np.array_equal(w.view(np.uint32), g["w"][k].view(np.uint32))
        assert np.array_equal(y.view(np.uint32), g["y"][k].view(np.uint32))


@pytest.mark.parametrize("T", [3, 6])
def test_port_reproduces_prefill_fixture(T):
    g = load(f"prefill_e32_t{T}.npz")
    y, idx, w = oracle.moe_prefill(decode_layer(), g["x"], isa=ISA, impl="port")
    assert np.array_equal(idx, g["idx"])
    assert np.array_equal(w.view(np.uint32), g["w"].view(np.uint32))
    assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32))


def test_port_reproduces_forward_fixture():
    g = load("forward_e32_l2.npz")
    y = oracle.forward(forward_layers(), g["x"], isa=ISA, impl="port")
    assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32))


def _rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b)))


@pytest.mark.gpu
def test_gpu_decode_matches_fixture():
    import ttl_moe
    g = load("decode_e32.npz")
    with ttl_moe.MoE(experts=32, layers=1, device=0) as m:
        m.upload_layer(0, decode_layer())
        for k in range(g["x"].shape[0]):
            y, idx, w = m.moe(0, g["x"][k])
            assert np.array_equal(idx, g["idx"][k])
            np.testing.assert_allclose(w, g["w"][k], rtol=1e-5)
            assert _rel(y, g["y"][k]) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("T", [3, 6])
def test_gpu_prefill_matches_fixture(T):
    import ttl_moe
    g = load(f"prefill_e32_t{T}.npz")
    with ttl_moe.MoE(experts=32, layers=1, max_tokens=8, device=0) as m:
        m.upload_layer(0, decode_layer())
        y, idx, w = m.moe_batch(0, g["x"])
    assert np.array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["w"], rtol=1e-5)
    for k in range(T):
        assert _rel(y[k], g["y"][k]) <= TOL


@pytest.mark.gpu
def test_gpu_forward_matches_fixture():
    import ttl_moe
    g = load("forward_e32_l2.npz")
    with ttl_moe.MoE(experts=32, layers=2, device=0) as m:
        for l, t in enumerate(forward_layers()):
            m.upload_layer(l, t)
        y = m.forward(0, 2, g["x"])
    for k in range(y.shape[0]):
        assert _rel(y[k], g["y"][k]) <= TOL
