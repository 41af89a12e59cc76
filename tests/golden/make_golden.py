"""Writes the golden fixtures of the MoE path from tt-lab's own compiled code.

Run from the repository root after `make -C oracle ref` (needs the reference
sources, so it runs where they are, not on the GPU box):

    python tests/golden/make_golden.py

Each fixture holds the seeded synthetic layer's generator parameters (the
423 MB of weights are regenerated from them by ttl_moe.synth, whose output is
pinned by tests/test_synth.py), the exact inputs, and the outputs of the
compiled reference (oracle/_ref: tt-lab src/tensor.cpp, src/gguf.cpp and
src/model.cpp built unmodified, driven through GptOssModel::moe / moe_batch).
"""
from __future__ import annotations

import json
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))

import oracle  # noqa: E402
from ttl_moe import synth  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent


def main() -> int:
    if not oracle.ref_available():
        print("reference oracle not built (make -C oracle ref)", file=sys.stderr)
        return 1
    isa = "x86-64-v4" if oracle.ref().tref_isa_v4() else "default"
    meta = {"generator": "tests/golden/make_golden.py", "reference_clone": isa, "fixtures": {}}

    # decode, gpt-oss-20b shapes: layer (seed 7, layer 3, 32 experts), 3 tokens
    t = synth.layer_host(7, 3, 32)
    x = synth.inputs_host(11, 3)
    ys, idxs, ws = [], [], []
    for k in range(3):
        y, idx, w = oracle.moe_decode(t, x[k], impl="ref")
        ys.append(y), idxs.append(idx), ws.append(w)
    np.savez_compressed(HERE / "decode_e32.npz", x=x, y=np.stack(ys), idx=np.stack(idxs), w=np.stack(ws))
    meta["fixtures"]["decode_e32.npz"] = {"layer": {"seed": 7, "layer": 3, "experts": 32},
                                          "call": "GptOssModel::moe per token"}

    # prefill: T = 3 (matvec route, src/model.cpp:404-411) and T = 6 (matmul route, :413-420)
    for T in (3, 6):
        xb = synth.inputs_host(13, T)
        y, idx, w = oracle.moe_prefill(t, xb, impl="ref")
        np.savez_compressed(HERE / f"prefill_e32_t{T}.npz", x=xb, y=y, idx=idx, w=w)
        meta["fixtures"][f"prefill_e32_t{T}.npz"] = {"layer": {"seed": 7, "layer": 3, "experts": 32},
                                                     "call": "GptOssModel::moe_batch"}

    # layer stack: 2 layers with RMSNorm weights, 2 tokens (x <- x + moe(rms_norm(x) * g))
    layers = [synth.layer_host(21, l, 32, norm=True) for l in range(2)]
    xs = synth.inputs_host(23, 2)
    yf = oracle.forward(layers, xs, impl="ref")
    np.savez_compressed(HERE / "forward_e32_l2.npz", x=xs, y=yf)
    meta["fixtures"]["forward_e32_l2.npz"] = {"layers": [{"seed": 21, "layer": l, "experts": 32, "norm": True}
                                                         for l in range(2)],
                                              "call": "rms_norm + GptOssModel::moe + residual per layer"}

    (HERE / "golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(json.dumps(meta))
    return 0


if __name__ == "__main__":
    sys.exit(main())
