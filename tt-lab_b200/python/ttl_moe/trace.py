"""Per-phase timeline of the persistent decode kernel (ttl_moe_trace).

    python -m ttl_moe.trace [--experts 32] [--layers 24] [--tokens 256]

Builds a handle with seeded synthetic layers in device memory (the
benchmark's cfg1 shapes by default), runs ``forward`` over all tokens x
layers in one launch, and prints, per traced step, the %globaltimer stamps of
CTA 0 relative to the step's start, plus the latest CTA's gate/up and down
ends.  One JSON line: the launch's time per token-layer and, per point, its
mean / median / p90 in microseconds (the first steps are skipped as warm-up).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

# stamp index -> meaning (decode_tc.cu, `stamp`)
POINTS = {
    0: "step_start",
    4: "router_sums_in",
    1: "selection_published",
    2: "gateup_operand_ready",
    3: "cta0_gateup_done",
    8: "latest_gateup_done",
    5: "down_operand_ready",
    6: "cta0_down_done",
    9: "latest_down_done",
    7: "step_end",
}


def phase_table(trace: np.ndarray, skip: int) -> dict:
    """Mean / median / p90 (us) of every stamp relative to its step's start."""
    tr = trace.astype(np.float64)
    rel = (tr - tr[:, :1]) / 1e3
    steps = np.diff(tr[:, 0]) / 1e3
    rows = slice(skip, tr.shape[0] - 1)
    out = {"step_us": {"mean": float(steps[rows].mean()), "median": float(np.median(steps[rows]))}}
    for i, name in POINTS.items():
        v = rel[rows, i]
        out[name] = {"mean": round(float(v.mean()), 3), "median": round(float(np.median(v)), 3),
                     "p90": round(float(np.percentile(v, 90)), 3)}
    return out


def run(experts=32, layers=24, tokens=256, seed=0, trace_steps=1024):
    import torch

    from . import MoE, synth
    torch.cuda.set_device(0)
    m = MoE(experts=experts, layers=layers, max_tokens=0, device=0)
    try:
        for l in range(layers):
            t = synth.layer_device(seed, l, experts, device="cuda")
            m.upload_layer(l, t)
            del t
        torch.cuda.empty_cache()
        x = torch.from_numpy(synth.inputs_host(seed, tokens)).cuda()
        y = torch.empty_like(x)
        st = torch.cuda.ExternalStream(m.stream())
        for _ in range(3):
            m.forward_async(0, layers, x, y, tokens)
        m.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(5):
            m.forward_async(0, layers, x, y, tokens)
        e1.record(st)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / 5
        n = min(trace_steps, tokens * layers)
        m.trace_enable(n)
        m.forward_async(0, layers, x, y, tokens)
        m.sync()
        table = phase_table(m.trace(), skip=min(48, n // 4))
    finally:
        m.close()
    return {"experts": experts, "layers": layers, "tokens": tokens, "traced_steps": n,
            "us_per_token_layer_untraced": ms * 1e3 / (tokens * layers), "phases_us": table}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--experts", type=int, default=32)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--tokens", type=int, default=256)
    args = ap.parse_args(argv)
    print(json.dumps(run(args.experts, args.layers, args.tokens)))


if __name__ == "__main__":
    main()
