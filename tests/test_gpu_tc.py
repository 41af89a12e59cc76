"""Tensor-core MXFP4 matvec (ttl_matvec_mxfp4) against tt-lab's
matvec_add_mxfp4_2880 (src/tensor.cpp:239-304) restated in the oracle, and
against the reference's own known answer (tests/host_dispatch.cpp:92-107)."""
import numpy as np
import pytest

import oracle
from conftest import synth_layer

pytestmark = pytest.mark.gpu
D = 2880
EXPERT = D * 90 * 17


def run(packed_host_gguf, bias, x):
    import torch
    import ttl_moe
    g = torch.from_numpy(packed_host_gguf).cuda()
    packed = torch.empty(ttl_moe.packed_bytes(1), dtype=torch.uint8, device="cuda")
    ttl_moe.pack_mxfp4(g, 1, packed)
    b = torch.from_numpy(bias).cuda()
    xx = torch.from_numpy(x).cuda()
    y = torch.empty(D, dtype=torch.float32, device="cuda")
    ttl_moe.matvec_mxfp4(packed, b, xx, y)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_tc_matvec_known_answer():
    data = np.zeros(EXPERT, np.uint8)
    blocks = data.reshape(-1, 17)
    blocks[:, 0] = 127
    blocks[:, 1:] = 0x21
    y = run(data, np.full(D, 0.25, np.float32), np.full(D, 0.5, np.float32))
    assert np.all(y == np.float32(1080.25)), (y[:4], y[-4:])


@pytest.mark.parametrize("which", ["gate_w", "down_w"])
def test_tc_matvec_matches_oracle(which):
    from ttl_moe import synth
    t = synth_layer(0, 32)
    w = np.ascontiguousarray(t[which][3 * EXPERT:4 * EXPERT])
    bias = np.ascontiguousarray(t["gate_b"][3 * D:4 * D])
    x = synth.inputs_host(5, 1)[0] * np.float32(3.0)
    ref = np.empty(D, np.float32)
    oracle.port().oref_matvec_add_mxfp4(w.ctypes.data, bias.ctypes.data, x.ctypes.data, ref.ctypes.data,
                                        oracle.ISA_DEFAULT)
    y = run(w, bias, x)
    m = oracle.compare(y, ref)
    assert m["max_rel"] <= 1e-4, m
