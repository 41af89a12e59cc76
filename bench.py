#!/usr/bin/env python3
"""Benchmark of the B200 gpt-oss MoE path.

Workload (one "step"): gpt-oss-20b 24-layer MoE stack, decode T = 1 for 256
sequential tokens; per token and layer h = RMSNorm(x), x = x + MoE(h)
(tt-lab src/model.cpp:590-594 without attention).  Weights are seeded synthetic
MXFP4 (csrc/synth.h), 10.2 GB of experts resident in HBM, so every token streams
1.28 GB and no step can be served from the 126 MB L2.

The line also carries "prefill": BASELINE.json configs[2] (one gpt-oss-20b
layer, T = 512, Zipf(1.1)-skewed routing) through the same library, timed with
CUDA events; --prefill-only runs just that part.

Arms
  default            libttl_moe through its C ABI (this repo's kernels).
  --impl reference   tt-lab's own CPU MoE (GptOssModel::moe, compiled from its
                     sources into oracle/_ref) on the host cores, bounded sample.

Multi-GPU (torchrun, N > 1): expert parallel -- experts sharded E/N per rank,
router replicated, NCCL all-reduce of the partial outputs per layer; the same
256 tokens are processed by the job ("strong" scaling).  Timing: barrier +
synchronize on both sides, CUDA events on the library's stream, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))

DIM = 2880
GGUF_MATRIX = 2880 * 90 * 17            # 4,406,400 B per expert matrix
BIAS = 2880 * 4
# Algorithmic bytes of one decode MoE layer (E = 32): router W + bias, 12 expert
# matrices + their biases, input and output vectors.
LAYER_BYTES_20B = 32 * DIM * 4 + 32 * 4 + 12 * GGUF_MATRIX + 12 * BIAS + 2 * DIM * 4
# The gate/up kernel of one layer: 8 matrices + 8 bias rows + h in + 4 hidden rows out.
GATEUP_BYTES = 8 * GGUF_MATRIX + 8 * BIAS + DIM * 4 + 4 * DIM * 4


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.gpu], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_reference_sample(experts, seconds, threads, seed=0):
    """tt-lab's own GptOssModel::moe on host cores for ~`seconds` on one
    seeded layer (423 MB of experts, far above the LLC) and a stream of
    seeded tokens.  Returns (token-layers per second, calls, elapsed, isa)."""
    import oracle
    from oracle import synth as osynth
    t = osynth.layer_host(seed, 0, experts)
    xs = osynth.inputs_host(seed, 64)
    out = np.empty(DIM, np.float32)
    R = oracle.ref()
    args = [t[n].ctypes.data for n in ("router_w", "router_b", "gate_w", "gate_b", "up_w", "up_b", "down_w",
                                        "down_b")]
    # one untimed call (page-in)
    oracle.moe_decode(t, xs[0], impl="ref")
    calls = 0
    t0 = time.perf_counter()
    while True:
        x = xs[calls % xs.shape[0]]
        if threads <= 1:
            rc = R.tref_moe_decode(experts, *args, x.ctypes.data, out.ctypes.data, None, None)
        else:
            rc = R.tref_moe_decode_threaded(experts, *args, x.ctypes.data, out.ctypes.data, threads)
        if rc != 0:
            raise RuntimeError(R.tref_last_error().decode())
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return calls / el, calls, el, ("x86-64-v4" if R.tref_isa_v4() else "default")


def cfg1_config(layers, tokens):
    """The workload both arms name (identical dict in both JSON lines)."""
    return {"workload": "cfg1: gpt-oss-20b 24-layer MoE stack, decode T=1, 256 sequential tokens",
            "experts": 32, "layers": layers, "tokens_per_step": tokens,
            "l2": "inputs larger than L2: 1.28 GB of expert weights streamed per token",
            "weights": "MXFP4 (E2M1 + E8M0 per 32), f32 activations and accumulation"}


def run_reference(args, world, rank):
    """--impl reference: tt-lab's own CPU decode path (GptOssModel::moe with
    rms_norm and the residual, compiled from its sources into oracle/_ref) on
    all host threads.  The 256 tokens are independent sequences, so the
    threads run them side by side, one token per thread through all 24
    layers (each token's arithmetic is the single-threaded reference's).  A
    step is one such round: `threads` of the 256 tokens (a bounded sample of
    the workload), timed as it runs.  Inputs come from the oracle's own
    generator (the same seeded tensors as the GPU arm); the product library is
    never loaded in this process."""
    layers, tokens = args.layers, args.tokens
    if rank != 0:
        return 0
    try:
        import oracle
        from oracle import synth as osynth
        oracle.ref()
    except OSError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU path not built: {e}"}))
        return 0
    threads = max(1, os.cpu_count() or 1)
    per_step = max(1, min(tokens, threads))
    t0 = time.perf_counter()
    weights = [osynth.layer_host(0, l, 32) for l in range(layers)]
    x = osynth.inputs_host(0, tokens)
    gen_s = time.perf_counter() - t0
    times = []
    for i in range(args.warmup + args.steps):
        lo = (i * per_step) % tokens
        idx = [(lo + j) % tokens for j in range(per_step)]
        xs = np.ascontiguousarray(x[idx])
        t1 = time.perf_counter()
        oracle.forward_tokens(weights, xs, threads=threads)
        dt = time.perf_counter() - t1
        if i >= args.warmup:
            times.append(dt)
    step_s = statistics.median(times)
    value = per_step / step_s
    isa = "x86-64-v4" if oracle.ref().tref_isa_v4() else "default"
    line = {
        "metric": "MoE decode tokens/s (gpt-oss-20b, 24 MoE layers, T=1)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "impl": "reference",
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; BASELINE.json cfg1 "
        "distributions, the GPU arm's tensors)", "parallelism": f"{threads} host threads, one token each",
        "config": cfg1_config(layers, tokens),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"each step: {per_step} of the {tokens} tokens, one per host thread, through "
                                   f"all {layers} layers with tt-lab's GptOssModel::moe + rms_norm + residual "
                                   f"({isa} clone); median of {args.steps} timed steps ({step_s * 1e3:.0f} ms "
                                   f"each) after {args.warmup} warm-up; inputs generated in {gen_s:.1f}s before "
                                   "timing"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def decode_parity_sample(torch, moe, synth, x_host, y_timed, layers, tokens=16, seed=0):
    """Parity of the headline launch on a sample, after the timed region: the
    first `tokens` of the 256 tokens go through the same forward launch again
    with the step log on (their outputs must equal the timed run's bit for
    bit: the kernel is deterministic and tokens are independent), and each of
    their tokens x layers steps is replayed through tt-lab's compiled CPU code
    on the GPU's own input for it (oracle/parity.py)."""
    import oracle
    from oracle import parity
    steps = tokens * layers
    ylog = torch.empty((steps, DIM), dtype=torch.float32, device="cuda")
    ilog = torch.empty((steps, 4), dtype=torch.int32, device="cuda")
    wlog = torch.empty((steps, 4), dtype=torch.float32, device="cuda")
    moe.record(steps, ylog, ilog, wlog)
    xs = torch.from_numpy(np.ascontiguousarray(x_host[:tokens])).cuda()
    ys = torch.empty_like(xs)
    moe.forward_async(0, layers, xs, ys, tokens)
    moe.sync()
    moe.record(0)
    same = bool(torch.equal(ys, y_timed[:tokens]))
    yl = ylog.cpu().numpy().reshape(tokens, layers, DIM)
    il = ilog.cpu().numpy().reshape(tokens, layers, 4)
    wl = wlog.cpu().numpy().reshape(tokens, layers, 4)

    def layer_iter():
        for l in range(layers):
            t = synth.layer_device(seed, l, 32, device="cuda")
            yield l, {k: v.cpu().numpy() for k, v in t.items()}

    t0 = time.perf_counter()
    s = parity.teacher_forced(layer_iter(), x_host[:tokens], yl, il, wl)
    return {"passed": parity.passed(s) and same, "steps": s["steps"], "max_rel": s["max_rel"],
            "max_rel_bar": parity.TOL, "top4_mismatches": s["mismatches"], "near_ties": s["near_ties"],
            "top4_weights_max_rel": s["max_w_rel"], "identical_to_timed_run": same,
            "sample": f"tokens 0-{tokens - 1} of the 256 x all {layers} layers ({steps} steps), each step replayed "
                      "through tt-lab's compiled rms_norm + GptOssModel::moe + residual (oracle/_ref) on the "
                      f"GPU's own input for it; checked in {time.perf_counter() - t0:.1f}s after the timed region"}


# Dense FP4 tensor-core peak of one B200 (nominal; MEASURED_PEAKS.json has no FP4 figure).
FP4_PEAK_TFLOPS = 9000.0
PREFILL_DIGITS = 6      # radix-8 digit rows per activation (B operand of the prefill MMAs)
PREFILL_GROUP = 16      # slots per expert group (N = 16 x 6 = 96 per group)


def cpu_prefill_sample(seconds, seed=2, experts=32):
    """tt-lab's own GptOssModel::moe_batch (oracle/_ref, 1 thread) on the cfg2
    layer, on a bounded prefix of the cfg2 tokens sized to take about
    `seconds`.  Returns (tokens per second, tokens, elapsed, isa)."""
    import oracle
    from ttl_moe import synth
    t = synth.layer_host(seed, 0, experts, zipf_s=1.1)
    x = synth.inputs_host(seed, 512)
    oracle.moe_prefill(t, x[:4], impl="ref")  # page-in
    t0 = time.perf_counter()
    oracle.moe_prefill(t, x[:8], impl="ref")
    per_token = (time.perf_counter() - t0) / 8
    n = int(min(512, max(8, seconds / max(per_token, 1e-6))))
    t0 = time.perf_counter()
    oracle.moe_prefill(t, x[:n], impl="ref")
    el = time.perf_counter() - t0
    R = oracle.ref()
    return n / el, n, el, ("x86-64-v4" if R.tref_isa_v4() else "default")


def prefill_cfg2(torch, ttl_moe, synth, device, iters=20, cpu_seconds=0.0):
    """one gpt-oss-20b layer, prefill T = 512, router
    bias Zipf(1.1)-skewed.  Device time per layer (CUDA events on the library's
    stream, 425 MB of experts per layer > L2), the host-buffer call end to end,
    and the MXFP4 MMA work the grouped kernels execute.  The end-to-end figure
    is the host-buffer call (ttl_moe_prefill) on pinned buffers: H2D of x, the
    kernels, D2H of the output and the top-4 indices and weights."""
    import numpy as np
    T, E = 512, 32
    with ttl_moe.MoE(experts=E, layers=1, max_tokens=T, device=device) as m:
        m.upload_layer(0, synth.layer_device(2, 0, E, device="cuda", zipf_s=1.1))
        xh = synth.inputs_host(2, T)
        x = torch.from_numpy(xh).cuda()
        out = torch.empty_like(x)
        st = torch.cuda.ExternalStream(m.stream())
        for _ in range(3):
            m.prefill_async(0, x, T, out)
        m.sync()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(iters):
            m.prefill_async(0, x, T, out)
        e1.record(st)
        e1.synchronize()
        m.sync()
        ms = e0.elapsed_time(e1) / iters
        pout, idx, _ = m.moe_batch(0, xh)
        x_pin = torch.from_numpy(xh).pin_memory()
        o_pin = torch.empty_like(x_pin).pin_memory()
        i_pin = torch.empty((T, 4), dtype=torch.int32).pin_memory()
        w_pin = torch.empty((T, 4), dtype=torch.float32).pin_memory()
        m.prefill_host(0, x_pin, T, o_pin, i_pin, w_pin)
        t0 = time.perf_counter()
        for _ in range(iters):
            m.prefill_host(0, x_pin, T, o_pin, i_pin, w_pin)
        e2e_ms = (time.perf_counter() - t0) / iters * 1e3
    cpu = None
    if cpu_seconds > 0:
        try:
            rate, n, el, isa = cpu_prefill_sample(cpu_seconds)
            cpu = {"value": rate, "unit": "tokens/s", "cores": 1, "kind": "reference",
                   "sample": f"GptOssModel::moe_batch on the first {n} cfg2 tokens ({el:.1f}s, 1 thread, {isa} clone)"}
        except Exception as e:  # the reference build is optional on the box
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    parity = None
    try:
        import oracle
        th = synth.layer_host(2, 0, E, zipf_s=1.1)
        t0 = time.perf_counter()
        rout, ridx, _ = oracle.moe_prefill(th, xh, impl="ref")
        bad = int(np.count_nonzero(np.any(np.asarray(idx) != ridx, axis=1)))
        good = np.all(np.asarray(idx) == ridx, axis=1)
        mm = oracle.compare(pout[good], rout[good])
        parity = {"passed": bad == 0 and mm["max_rel"] <= 1e-3, "tokens": T, "max_rel": mm["max_rel"],
                  "top4_mismatches": bad,
                  "sample": f"all {T} tokens against tt-lab's GptOssModel::moe_batch (oracle/_ref, 1 thread, "
                            f"{time.perf_counter() - t0:.1f}s), after the timed region"}
    except OSError as e:
        parity = {"passed": None, "sample": f"unavailable: {e}"}
    counts = np.bincount(np.asarray(idx).ravel(), minlength=E)
    groups = int(sum((c + PREFILL_GROUP - 1) // PREFILL_GROUP for c in counts))
    rows = (DIM + 127) // 128 * 128
    mma_flop = 3 * groups * PREFILL_GROUP * PREFILL_DIGITS * rows * DIM * 2
    useful_flop = 3 * T * 4 * DIM * DIM * 2
    return {
        "workload": "cfg2: gpt-oss-20b single MoE layer, prefill T=512, router bias Zipf(1.1)",
        "ms_per_layer": ms,
        "tokens_per_s": T / (ms * 1e-3),
        "e2e": {"ms_per_layer": e2e_ms, "tokens_per_s": T / (e2e_ms * 1e-3),
                "h2d_bytes_per_step": T * DIM * 4, "d2h_bytes_per_step": T * DIM * 4 + T * 4 * 8},
        "expert_groups": groups,
        "max_expert_pairs": int(counts.max()),
        "mma_tflops": mma_flop / (ms * 1e-3) / 1e12,
        "mma_frac_of_nominal_fp4": mma_flop / (ms * 1e-3) / 1e12 / FP4_PEAK_TFLOPS,
        "reference_math_tflops": useful_flop / (ms * 1e-3) / 1e12,
        "tensor_pipe_source": "profiles/prefill_mma_cfg2_T512.md (ncu sm__pipe_tensor_cycles_active)",
        "cpu_baseline": cpu,
        "parity": parity,
    }


VOCAB = 201088
HEAD_BYTES = VOCAB * 90 * 34 + VOCAB * 4 + 2 * DIM * 4  # Q8_0 output.weight, logits out, x + norm in


def logits_head(torch, ttl_moe, synth, hbm_peak, iters=20, cpu_seconds=6.0):
    """The output head of GptOssModel::forward (src/model.cpp:598-612): rms_norm
    with output_norm.weight, matvec_q8_0 over the 201,088 x 2880 Q8_0
    output.weight (615 MB, far above L2) and greedy, on seeded synthetic
    weights.  Device time per call (CUDA events on the head's stream, x and
    the logits in HBM), the host call end to end (x in, logits and token out),
    tt-lab's own rms_norm + matvec_q8_0 + greedy on one host thread, and the
    logits of two inputs checked bit for bit against it."""
    import oracle
    t = synth.head_device(0, VOCAB)
    xs = synth.inputs_host(9, 4)
    with ttl_moe.Head(vocab=VOCAB, device=torch.cuda.current_device()) as h:
        h.upload(t["output_w"], t["output_norm"])
        wh = t["output_w"].cpu().numpy()
        gh = t["output_norm"].cpu().numpy()
        del t
        torch.cuda.empty_cache()
        xd = torch.from_numpy(xs).cuda()
        ld = torch.empty(VOCAB, dtype=torch.float32, device="cuda")
        td = torch.empty(1, dtype=torch.int32, device="cuda")
        st = torch.cuda.ExternalStream(h.stream())
        for i in range(3):
            h.forward_async(xd[i % 4], ld, td)
        h.sync()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(iters):
            h.forward_async(xd[i % 4], ld, td)
        e1.record(st)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        h.forward(xs[0])
        t0 = time.perf_counter()
        for i in range(iters):
            logits, tok = h.forward(xs[i % 4])
        e2e_ms = (time.perf_counter() - t0) / iters * 1e3
        checks = []
        for i in range(2):
            gl, gt = h.forward(xs[i])
            rl, rt = oracle.head(wh, gh, xs[i], VOCAB, impl="ref")
            nan = np.isnan(rl)
            checks.append(bool(np.array_equal(np.isnan(gl), nan) and
                               np.array_equal(gl[~nan].view(np.uint32), rl[~nan].view(np.uint32)) and gt == rt))
    oracle.head(wh, gh, xs[0], VOCAB, impl="ref")
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < cpu_seconds or n == 0:
        oracle.head(wh, gh, xs[n % 4], VOCAB, impl="ref")
        n += 1
    cpu_ms = (time.perf_counter() - t0) / n * 1e3
    gbs = HEAD_BYTES / (ms * 1e-3) / 1e9
    return {"workload": "output head: rms_norm + matvec_q8_0 (201088 x 2880 Q8_0, 615 MB) + greedy, one token",
            "ms_per_call": ms, "tokens_per_s": 1e3 / ms,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "bytes_per_call": HEAD_BYTES,
                         "kernels": "head_norm_kernel + head_matvec_kernel, CUDA events around both"},
            "e2e": {"ms_per_call": e2e_ms, "h2d_bytes_per_step": DIM * 4, "d2h_bytes_per_step": VOCAB * 4 + 4},
            "cpu_baseline": {"value": 1e3 / cpu_ms, "unit": "tokens/s", "cores": 1, "kind": "reference",
                             "sample": f"{n} calls of tt-lab's rms_norm + matvec_q8_0 + greedy (oracle/_ref, 1 "
                                       f"thread), {cpu_ms:.1f} ms each"},
            "parity": {"passed": all(checks), "inputs": len(checks),
                       "what": "logits bit-equal to tt-lab's (NaN positions equal) and the same greedy token"}}


# Algorithmic bytes of one attention block at a given number of attended
# positions: Q8_0 Q / K / V (4096 + 512 + 512 rows of 2880) and output (2880
# rows of 4096), their biases, attn_norm and sinks, x in / residual out, the
# new K / V row written, and K / V of every attended position read (f32).
ATTN_WEIGHT_BYTES = (4096 + 512 + 512) * 90 * 34 + DIM * 128 * 34 + (4096 + 512 + 512 + DIM) * 4 + DIM * 4 + 64 * 4


def attn_bytes(attended):
    return ATTN_WEIGHT_BYTES + 2 * DIM * 4 + 2 * 512 * 4 + attended * 2 * 512 * 4


def attention_decode(torch, ttl_moe, synth, hbm_peak, context=1024, layers=24, iters=10):
    """The attention block of a 20b decode layer (src/model.cpp:572-590) on the
    GPU (ttl_attn), on seeded synthetic weights, at `context` positions
    already in the KV cache: device time per layer (CUDA events on the
    handle's stream over all `layers` layers of one token; even layers attend
    to 128 positions, odd ones to all), and a whole GPU-resident decode token
    -- per layer attention then the MoE half (rms_norm -> moe -> residual,
    ttl_moe_forward) on one stream, then the output head -- in tokens/s.
    Parity of the attention block: tests/test_gpu_attn.py."""
    dev = torch.cuda.current_device()
    attn_t = [synth.attention_layer_host(5, l) for l in range(layers)]
    with ttl_moe.MoE(experts=32, layers=layers, device=dev) as m, \
            ttl_moe.Attention(layers=layers, token_capacity=context + 2 * iters + 8, device=dev, stream=m.stream()) as a, \
            ttl_moe.Head(vocab=VOCAB, device=dev) as h:
        for l in range(layers):
            a.upload_layer(l, attn_t[l])
            t = synth.layer_device(0, l, 32, device="cuda")
            m.upload_layer(l, t)
            del t
        ht = synth.head_device(0, VOCAB)
        h.upload(ht["output_w"], ht["output_norm"])
        del ht
        torch.cuda.empty_cache()
        xs = torch.from_numpy(synth.inputs_host(11, 8)).cuda()
        buf = torch.empty((2, DIM), dtype=torch.float32, device="cuda")
        logits = torch.empty(VOCAB, dtype=torch.float32, device="cuda")
        tok = torch.empty(1, dtype=torch.int32, device="cuda")
        # fill the caches to `context` positions (attention only)
        for p in range(context):
            for l in range(layers):
                a.forward_async(l, p, xs[p % 8], buf[0])
        a.sync()
        st = torch.cuda.ExternalStream(m.stream())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p = context
        e0.record(st)
        for i in range(iters):
            for l in range(layers):
                a.forward_async(l, p, xs[i % 8], buf[0])
            p += 1
        e1.record(st)
        e1.synchronize()
        attn_ms = e0.elapsed_time(e1) / (iters * layers)
        # whole tokens: attention -> MoE half per layer, then the head (on
        # its own stream, after an event of the MoE stream)
        hst = torch.cuda.ExternalStream(h.stream())
        ev = torch.cuda.Event()

        def token(p):
            x = xs[p % 8]
            for l in range(layers):
                a.forward_async(l, p, x, buf[0])
                m.forward_async(l, l + 1, buf[0], buf[1], 1)
                x = buf[1]
            ev.record(st)
            hst.wait_event(ev)
            h.forward_async(x, logits, tok)
        token(p)
        p += 1
        h.sync()
        m.sync()
        t0 = time.perf_counter()
        for i in range(iters):
            token(p)
            p += 1
            h.sync()  # the head runs on its own stream; the next token's input waits for it
        tok_ms = (time.perf_counter() - t0) / iters * 1e3
        del hst
    avg_attended = (128 + context) / 2
    gbs = attn_bytes(avg_attended) / (attn_ms * 1e-3) / 1e9
    return {"workload": f"gpt-oss-20b attention block, {layers} layers, context {context} (even layers: window "
                        f"128), synthetic Q8_0 weights",
            "ms_per_layer": attn_ms,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "bytes_per_layer": attn_bytes(avg_attended),
                         "kernels": "attn_qkv_kernel + attn_decode_kernel + attn_out_kernel, CUDA events"},
            "decode_token": {"ms_per_token": tok_ms, "tokens_per_s": 1e3 / tok_ms,
                             "what": "one token through 24 x (attention + rms_norm -> MoE -> residual) and the "
                                     "output head, all on the GPU (wall clock per token, host waits for the "
                                     "greedy token)"}}


# Algorithmic bytes of one gpt-oss-120b decode token-layer (E = 128): router W
# + bias, 12 expert matrices + their biases, x / out.
LAYER_BYTES_120B = 128 * DIM * 4 + 128 * 4 + 12 * GGUF_MATRIX + 12 * BIAS + 2 * DIM * 4


def decode_cfg3(torch, ttl_moe, synth, local, world, rank, dist, tokens=64, steps=3):
    """gpt-oss-120b 36-layer MoE stack (128 experts,
    seeded synthetic weights, 61 GB packed), decode T = 1 for `tokens`
    sequential tokens, experts sharded E/N per rank with the in-kernel
    exchange of partial outputs.  CUDA events on the library's stream around
    `steps` forward launches, max over ranks."""
    from ttl_moe import parallel
    E, layers = 128, 36
    nid = None
    if world > 1:
        nid = parallel.share_bytes(dist, ttl_moe.nccl_id() if rank == 0 else None, ttl_moe.NCCL_ID_BYTES,
                                   device="cuda")
    with ttl_moe.MoE(experts=E, layers=layers, max_tokens=0, device=local, rank=rank, world=world,
                     nccl_id_bytes=nid) as m:
        for l in range(layers):
            t = synth.layer_device(3, l, E, device="cuda")
            m.upload_layer(l, t)
            del t
        torch.cuda.empty_cache()
        x = torch.from_numpy(synth.inputs_host(3, tokens)).cuda()
        y = torch.empty_like(x)
        st = torch.cuda.ExternalStream(m.stream())
        for _ in range(2):
            m.forward_async(0, layers, x, y, tokens)
        m.sync()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            m.forward_async(0, layers, x, y, tokens)
        e1.record(st)
        e1.synchronize()
        m.sync()
        ms = e0.elapsed_time(e1) / steps
        persistent = m.counters()["persistent_decode"]
        # the routing of one launch (the kernel's step log), for the bytes
        # each GPU streams: its own selected experts per step, plus the
        # replicated router and the row in / out
        n = tokens * layers
        y_log = torch.empty((n, DIM), dtype=torch.float32, device="cuda")
        idx_log = torch.empty((n, 4), dtype=torch.int32, device="cuda")
        w_log = torch.empty((n, 4), dtype=torch.float32, device="cuda")
        m.record(n, y_log, idx_log, w_log)
        m.forward_async(0, layers, x, y, tokens)
        m.sync()
        m.record(0)
        own = idx_log.cpu().numpy() // (E // world)
        del y_log
    if dist:
        ms = parallel.max_over_ranks(dist, [ms], device="cuda")[0]
    tps = tokens / (ms * 1e-3)
    per_rank = np.array([(own == r).sum() for r in range(world)], np.float64) * 3 * (GGUF_MATRIX + BIAS)
    per_rank += n * (E * DIM * 4 + E * 4 + 2 * DIM * 4)
    hbm = peaks()[0]
    busiest = float(per_rank.max())
    return {"workload": f"cfg3: gpt-oss-120b 36-layer MoE stack, decode T=1, {tokens} sequential tokens, "
                        f"experts sharded 128/{world} per GPU",
            "tokens_per_s": tps, "ms_per_step": ms, "n_gpus": world, "persistent_kernel": bool(persistent),
            "algorithmic_gbs": tps * layers * LAYER_BYTES_120B / 1e9,
            "bytes_per_token_layer": LAYER_BYTES_120B,
            "per_gpu_bytes_per_launch": [int(v) for v in per_rank],
            "roofline_busiest_gpu": {"bound": "hbm", "achieved": busiest / (ms * 1e-3) / 1e9, "peak": hbm,
                                     "unit": "GB/s", "frac": busiest / (ms * 1e-3) / 1e9 / hbm,
                                     "what": "bytes the most-loaded GPU streams per launch (its selected experts "
                                             "from the kernel's step log, the replicated router, rows in/out) "
                                             "over the launch time"},
            "timing": f"CUDA events on the library stream around {steps} launches of {tokens} tokens x {layers} "
                      "layers, max over ranks"}


def prefill_cfg4(torch, ttl_moe, synth, local, world, rank, dist, iters=10):
    """one gpt-oss-120b layer (128 experts), prefill
    of T = 2048 tokens with Zipf(1.2)-skewed routing, expert-parallel over the
    job's ranks: rank r passes tokens [r T / N, (r + 1) T / N), which go to
    their experts' owners and come back as weighted rows (peer stores into the
    ranks' receive blocks).  Time per call: CUDA events on the library's
    stream, max over ranks."""
    from ttl_moe import parallel
    E, T = 128, 2048
    lo, hi = rank * T // world, (rank + 1) * T // world
    nid = None
    if world > 1:
        nid = parallel.share_bytes(dist, ttl_moe.nccl_id() if rank == 0 else None, ttl_moe.NCCL_ID_BYTES,
                                   device="cuda")
    with ttl_moe.MoE(experts=E, layers=1, max_tokens=hi - lo, device=local, rank=rank, world=world,
                     nccl_id_bytes=nid) as m:
        t = synth.layer_device(4, 0, E, device="cuda", zipf_s=1.2)
        m.upload_layer(0, t)
        del t
        torch.cuda.empty_cache()
        x = torch.from_numpy(synth.inputs_host(4, T)[lo:hi].copy()).cuda()
        out = torch.empty_like(x)
        st = torch.cuda.ExternalStream(m.stream())
        for _ in range(3):
            m.prefill_async(0, x, hi - lo, out)
        m.sync()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(iters):
            m.prefill_async(0, x, hi - lo, out)
        e1.record(st)
        e1.synchronize()
        m.sync()
        ms = e0.elapsed_time(e1) / iters
        # the routing of the call, for the bytes each GPU streams: the local
        # experts any token selects (each read once), the token rows it
        # receives and the weighted rows it returns
        idx_d = torch.empty((hi - lo, 4), dtype=torch.int32, device="cuda")
        m.prefill_async(0, x, hi - lo, out, idx_d)
        m.sync()
        owner = idx_d.long() // (E // world)
        active = torch.zeros(E, dtype=torch.int32, device="cuda")
        active[idx_d.long().flatten()] = 1
        rows = torch.zeros(world, dtype=torch.int64, device="cuda")
        pairs = torch.zeros(world, dtype=torch.int64, device="cuda")
        for r in range(world):
            hit = (owner == r)
            rows[r] = hit.any(dim=1).sum()
            pairs[r] = hit.sum()
        if dist:
            dist.all_reduce(active, op=dist.ReduceOp.MAX)
            dist.all_reduce(rows)
            dist.all_reduce(pairs)
        act = active.view(world, E // world).sum(dim=1).cpu().numpy().astype(np.float64)
        per_rank = act * 3 * (GGUF_MATRIX + BIAS) + (rows.cpu().numpy() + pairs.cpu().numpy()) * DIM * 4.0
    if dist:
        ms = parallel.max_over_ranks(dist, [ms], device="cuda")[0]
    hbm = peaks()[0]
    busiest = float(per_rank.max())
    return {"workload": "cfg4: gpt-oss-120b single MoE layer, prefill T=2048, router bias Zipf(1.2), "
                        f"expert-parallel over {world} GPU(s), tokens sharded T/N per rank",
            "ms_per_layer": ms, "tokens_per_s": T / (ms * 1e-3), "n_gpus": world,
            "per_gpu_bytes": [int(v) for v in per_rank],
            "roofline_busiest_gpu": {"bound": "hbm", "achieved": busiest / (ms * 1e-3) / 1e9, "peak": hbm,
                                     "unit": "GB/s", "frac": busiest / (ms * 1e-3) / 1e9 / hbm,
                                     "what": "bytes the most-loaded GPU streams per call (its active experts' "
                                             "weights once, received token rows, returned rows) over the call "
                                             "time"},
            "timing": "CUDA events on the library stream around 10 calls, max over ranks"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity sample checked after timing")
    ap.add_argument("--no-head", action="store_true", help="skip the output-head (logits) measurement")
    ap.add_argument("--no-120b", action="store_true", help="skip the cfg3 (120b, 36-layer) decode line")
    ap.add_argument("--no-attention", action="store_true",
                    help="skip the attention block / GPU-resident decode token measurement")
    ap.add_argument("--attention-only", action="store_true",
                    help="run only the attention block / decode-token measurement (profiling)")
    ap.add_argument("--attention-context", type=int, default=1024,
                    help="positions already in the KV cache for the attention measurement")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only the cfg2 prefill measurement (one JSON line with its figures)")
    args = ap.parse_args()

    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import numpy as np
    import torch
    import ttl_moe
    from ttl_moe import parallel, synth

    torch.cuda.set_device(local)
    if args.attention_only:
        if rank == 0:
            at = attention_decode(torch, ttl_moe, synth, peaks()[0], context=args.attention_context,
                                  iters=max(1, args.steps))
            print(json.dumps({"metric": "attention block ms/layer (gpt-oss-20b)", "value": at["ms_per_layer"],
                              "unit": "ms", "n_gpus": 1, "higher_is_better": False, "attention": at}))
        return 0
    if args.prefill_only:
        if rank == 0:
            pf = prefill_cfg2(torch, ttl_moe, synth, local, iters=max(1, args.steps),
                              cpu_seconds=0.0 if args.no_cpu_baseline else min(args.cpu_seconds, 6.0))
            print(json.dumps({"metric": "MoE prefill tokens/s (gpt-oss-20b layer, T=512)", "value": pf["tokens_per_s"],
                              "unit": "tokens/s", "n_gpus": 1, "higher_is_better": True, "prefill": pf}))
        return 0
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    experts, layers, tokens = 32, args.layers, args.tokens

    # NCCL id for the library's own communicator, broadcast over torch.distributed.
    nid = None
    if world > 1:
        nid = parallel.share_bytes(dist, ttl_moe.nccl_id() if rank == 0 else None, ttl_moe.NCCL_ID_BYTES,
                                   device="cuda")

    moe = ttl_moe.MoE(experts=experts, layers=layers, max_tokens=0, device=local, rank=rank, world=world,
                      nccl_id_bytes=nid)
    for l in range(layers):
        t = synth.layer_device(0, l, experts, device="cuda")
        moe.upload_layer(l, t)
        del t
    torch.cuda.empty_cache()

    x_host = synth.inputs_host(0, tokens)
    x_dev = torch.from_numpy(x_host).cuda()
    y_dev = torch.empty_like(x_dev)
    stream = torch.cuda.ExternalStream(moe.stream())
    moe.profile(True)

    def step():
        moe.forward_async(0, layers, x_dev, y_dev, tokens)

    for _ in range(max(3, args.warmup)):
        step()
    moe.sync()
    l0 = moe.counters()["launches"]

    clocks = ClockSampler(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)  # let the sampler start before the timed region
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    moe.sync()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    kms = moe.kernel_ms()
    launches = moe.counters()["launches"] - l0

    # e2e: the public host-buffer call with pinned buffers, H2D + D2H inside.
    x_pin = torch.from_numpy(x_host).pin_memory()
    y_pin = torch.empty_like(x_pin).pin_memory()
    moe.forward_host(0, layers, x_pin, y_pin, tokens)  # warm-up (captures its graph)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        moe.forward_host(0, layers, x_pin, y_pin, tokens)
    e2e_s = time.perf_counter() - t0
    if dist:
        dist.barrier()
    clk = clocks.stop()

    # the drop-in call of tt-lab's GptOssModel::moe: one (token, layer) per
    # blocking ttl_moe_decode on host buffers (H2D, one launch, D2H, sync)
    # (the C function called directly on preallocated buffers, so the figure
    # is the library call's and not Python's array handling)
    calls = 200
    xh = np.ascontiguousarray(x_host[0])
    oh = np.empty(DIM, np.float32)
    ih = np.empty(4, np.int32)
    wh = np.empty(4, np.float32)
    decode_fn = ttl_moe.lib().ttl_moe_decode
    hptr, xa, oa, ia, wa = moe.h, xh.ctypes.data, oh.ctypes.data, ih.ctypes.data, wh.ctypes.data
    ttl_moe.check(decode_fn(hptr, 0, xa, oa, ia, wa), hptr)
    if dist:
        dist.barrier()
    bad = 0
    t0 = time.perf_counter()
    for i in range(calls):
        bad |= decode_fn(hptr, i % layers, xa, oa, ia, wa)
    call_us = (time.perf_counter() - t0) / calls * 1e6
    ttl_moe.check(bad, hptr)
    # the same calls answered by a resident decode server (ttl_moe_serve),
    # single-GPU handles only
    serve_us = None
    if world == 1:
        moe.serve(100000)
        for i in range(20):
            bad |= decode_fn(hptr, i % layers, xa, oa, ia, wa)
        t0 = time.perf_counter()
        for i in range(calls):
            bad |= decode_fn(hptr, i % layers, xa, oa, ia, wa)
        serve_us = (time.perf_counter() - t0) / calls * 1e6
        ttl_moe.check(bad, hptr)
        moe.serve(0)
    if dist:
        call_us = parallel.max_over_ranks(dist, [call_us], device="cuda")[0]

    if dist:
        ms, e2e_s = parallel.max_over_ranks(dist, [ms, e2e_s], device="cuda")

    parity = None
    if world == 1 and not args.no_parity:
        try:
            parity = decode_parity_sample(torch, moe, synth, x_host, y_dev, layers)
        except OSError as e:  # the checker is not built on this machine
            parity = {"passed": None, "sample": f"unavailable: {e}"}

    ms_step = ms / args.steps
    value = tokens / (ms_step / 1e3)
    e2e_value = tokens * args.steps / e2e_s
    hbm_peak, peak_kind = peaks()
    if kms["persistent"]:
        kernel = "decode_tc_kernel"
        bytes_launch = LAYER_BYTES_20B * kms["steps"]
    else:  # expert-parallel handles: the gate/up kernel of one layer
        kernel = "decode_gateup_kernel"
        bytes_launch = GATEUP_BYTES
    kernel_gbs = bytes_launch / (kms["ms"] * 1e-3) / 1e9
    # DRAM traffic of the persistent kernel per token-layer, from the committed
    # ncu capture of a smaller stack (traffic grows with the token-layers).
    traffic = None
    prof = ROOT / "profiles" / "decode_tc_small_6x8.md"
    if kms["persistent"] and kernel == "decode_tc_kernel" and prof.exists():
        for ln in prof.read_text().splitlines():
            if ln.startswith("traffic_bytes_per_token_layer:"):
                traffic = int(ln.split(":")[1]) * kms["steps"]
    prefill = None
    prefill_ep = None
    if not args.no_prefill:
        moe.close()
        torch.cuda.empty_cache()
        if world == 1:
            prefill = prefill_cfg2(torch, ttl_moe, synth, local,
                                   cpu_seconds=0.0 if args.no_cpu_baseline else min(args.cpu_seconds, 6.0))
        prefill_ep = prefill_cfg4(torch, ttl_moe, synth, local, world, rank, dist)
    head = None
    if world == 1 and not args.no_head:
        moe.close()
        torch.cuda.empty_cache()
        try:
            head = logits_head(torch, ttl_moe, synth, peaks()[0],
                               cpu_seconds=0.0 if args.no_cpu_baseline else 6.0)
        except OSError as e:  # the checker is not built on this machine
            head = {"unavailable": str(e)}
    attention = None
    if world == 1 and not args.no_attention:
        moe.close()
        torch.cuda.empty_cache()
        attention = attention_decode(torch, ttl_moe, synth, peaks()[0], context=args.attention_context)
    decode_120b = None
    if not args.no_120b:
        moe.close()
        torch.cuda.empty_cache()
        decode_120b = decode_cfg3(torch, ttl_moe, synth, local, world, rank, dist)

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            try:
                rate, calls, el, isa = cpu_reference_sample(experts, args.cpu_seconds, 1)
                cpu = {"value": rate / layers, "unit": "tokens/s", "cores": 1, "kind": "reference",
                       "sample": f"{calls} GptOssModel::moe calls ({el:.1f}s, 1 thread, {isa} clone) on one "
                                 f"423 MB layer; tokens/s = calls/s / {layers} layers"}
            except Exception as e:  # the reference build is optional on the box
                cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                       "sample": f"unavailable: {e}"}
        line = {
            "metric": "MoE decode tokens/s (gpt-oss-20b, 24 MoE layers, T=1)",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded; BASELINE.json cfg1 distributions)",
            "parallelism": f"ep{world}",
            "config": cfg1_config(layers, tokens),
            "hbm_gbs_step": LAYER_BYTES_20B * layers * value / 1e9,
            "roofline": {
                "bound": "hbm",
                "kernel": kernel,
                "achieved": kernel_gbs,
                "peak": hbm_peak,
                "unit": "GB/s",
                "frac": kernel_gbs / hbm_peak,
                "peak_kind": peak_kind,
                "traffic": traffic,
                "traffic_source": "profiles/decode_tc_small_6x8.md (ncu dram bytes per token-layer x token-layers)",
                "bytes_per_launch": bytes_launch,
                "bytes_per_token_layer": LAYER_BYTES_20B,
                "launch_ms": kms["ms"],
                "token_layers_per_launch": kms["steps"],
            },
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": tokens * DIM * 4,
                    "d2h_bytes_per_step": tokens * DIM * 4},
            "gpu_launches": launches,
            "decode_call": {"us_per_call": call_us, "calls": calls,
                            "us_per_call_served": serve_us,
                            "what": "ttl_moe_decode (tt-lab's GptOssModel::moe drop-in): one token-layer per "
                                    "blocking call on host buffers, wall clock, max over ranks; 'served': the "
                                    "same calls answered by a resident decode kernel (ttl_moe_serve)"},
            "prefill": prefill,
            "prefill_ep": prefill_ep,
            "logits_head": head,
            "attention": attention,
            "decode_120b": decode_120b,
        }
        print(json.dumps(line))
    moe.close()
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
