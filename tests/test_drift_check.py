"""Drift report of the CUDA MoE path against tt-lab's CPU MoE, in the form of
tt-lab's `--device-proxy --check` (run_device_proxy_check,
src/tt_backend.cpp:3647-3714; metrics compare_vectors :3100-3128,
expert_overlap :3149-3159).

Per token and layer, the MoE of the same normalized input on the GPU and on
the CPU: rel RMS and cosine of the outputs, top-4 overlap and top-1 match of
the selected experts.  Per token, the residual stream after all layers
(ttl_moe_forward against the oracle's RMSNorm -> MoE -> residual chain).
Synthetic seeded layers stand in for a GGUF model.

    python tests/test_drift_check.py [tokens] [layers]     # prints the report
"""
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))
sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))

import oracle  # noqa: E402


def expert_overlap(a, b):
    return sum(1 for i in range(4) for j in range(4) if int(a[i]) == int(b[j]))


def run_check(tokens=4, layers=4, experts=32, seed=60, device=0, out=print):
    import ttl_moe
    from ttl_moe import synth
    from conftest import synth_layer
    impl = "ref" if oracle.ref_available() else "port"
    ls = [synth_layer(seed + l, experts, layer=l, norm=True) for l in range(layers)]
    xs = synth.inputs_host(seed + 100, tokens)
    stats = {"layers": 0, "overlap": 0, "top1": 0, "moe_rel_rms": 0.0, "moe_cos_min": 1.0,
             "x_rel_rms": [], "x_cos_min": 1.0}
    with ttl_moe.MoE(experts=experts, layers=layers, max_tokens=0, device=device) as m:
        for l, t in enumerate(ls):
            m.upload_layer(l, t)
        y = m.forward(0, layers, xs)
        for k in range(tokens):
            x = np.ascontiguousarray(xs[k])
            for l, t in enumerate(ls):
                h = oracle.rms_norm(x, t["norm_w"], impl=impl)
                g_out, g_idx, _ = m.moe(l, h)
                c_out, c_idx, _ = oracle.moe_decode(t, h, impl=impl)
                cm = oracle.compare(g_out, c_out)
                stats["layers"] += 1
                stats["overlap"] += expert_overlap(g_idx, c_idx)
                stats["top1"] += int(int(g_idx[0]) == int(c_idx[0]))
                stats["moe_rel_rms"] += cm["rel_rms"]
                stats["moe_cos_min"] = min(stats["moe_cos_min"], cm["cosine"])
                x = (x + c_out).astype(np.float32)
        ref = oracle.forward(ls, xs, impl=impl)
        for k in range(tokens):
            xm = oracle.compare(y[k], ref[k])
            stats["x_rel_rms"].append(xm["rel_rms"])
            stats["x_cos_min"] = min(stats["x_cos_min"], xm["cosine"])
            out(f"cuda check token {k + 1}/{tokens}: x cosine {xm['cosine']:.6f}, rel RMS {xm['rel_rms']:.6g}, "
                f"max abs {xm['max_abs']:.6g}")
    n = stats["layers"]
    worst = int(np.argmax(stats["x_rel_rms"]))
    out(f"x summary: avg rel RMS {np.mean(stats['x_rel_rms']):.6g}, max rel RMS {stats['x_rel_rms'][worst]:.6g} "
        f"at token {worst + 1}, min cosine {stats['x_cos_min']:.6f}")
    out(f"layer drift summary: MoE avg rel RMS {stats['moe_rel_rms'] / n:.6g} min cosine {stats['moe_cos_min']:.6f}")
    out(f"expert selection summary: avg top-4 overlap {stats['overlap'] / n:.3f}/4, top-1 match {stats['top1'] / n:.3f}")
    stats["overlap_avg"] = stats["overlap"] / n
    stats["top1_rate"] = stats["top1"] / n
    return stats


@pytest.mark.gpu
def test_drift_report_matches_reference():
    s = run_check(tokens=3, layers=3)
    assert s["overlap_avg"] == 4.0 and s["top1_rate"] == 1.0
    assert s["moe_cos_min"] > 0.999999 and s["moe_rel_rms"] / s["layers"] < 1e-5
    # the residual stream carries the f32 rounding of every layer (and the
    # forward path's f64 router sums); the parity bar is 1e-3
    assert s["x_cos_min"] > 0.99999 and max(s["x_rel_rms"]) < 1e-4


if __name__ == "__main__":
    run_check(tokens=int(sys.argv[1]) if len(sys.argv) > 1 else 4, layers=int(sys.argv[2]) if len(sys.argv) > 2 else 4)
