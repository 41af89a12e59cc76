"""The benchmark's seeded synthetic inputs, made on the CPU by the oracle's own
generator (oracle/synth_oracle.c) -- TEST INFRASTRUCTURE ONLY.

Same tensors, bit for bit, as the product library's generator
(tt-lab_b200/python/ttl_moe/synth.py; tests/test_synth.py holds the two
together), so the checker and bench.py's reference arm make their inputs
without loading the product library.  Distributions:

  router W [E][2880] ~ N(0, 0.02), router bias ~ N(0, 0.02) (+ optional Zipf shift)
  expert W  MXFP4 GGUF blocks: nibbles uniform over the 16 E2M1 codes, E8M0 scale
            bytes uniform over 119..125 (unbiased exponent -8..-2)
  expert biases ~ N(0, 0.02); activations ~ N(0, 1)
"""
from __future__ import annotations

import ctypes

import numpy as np

DIM = 2880
SCALE_LO = 119
SCALE_COUNT = 7
_KINDS = {"router_w": 0, "router_b": 1, "gate_w": 2, "gate_b": 3, "up_w": 4, "up_b": 5, "down_w": 6,
          "down_b": 7, "norm_w": 8, "zipf": 9}
INPUT_STREAM_BASE = 1 << 40
TENSORS = ("router_w", "router_b", "gate_w", "gate_b", "up_w", "up_b", "down_w", "down_b")


def stream(layer: int, name: str) -> int:
    return layer * 16 + _KINDS[name]


def _lib():
    from . import port
    L = port()
    if not getattr(L, "_synth_bound", False):
        u64, sz, vp = ctypes.c_uint64, ctypes.c_size_t, ctypes.c_void_p
        L.oref_synth_normal.argtypes = [vp, sz, u64, u64, ctypes.c_float, ctypes.c_float]
        L.oref_synth_normal.restype = None
        L.oref_synth_mxfp4.argtypes = [vp, sz, u64, u64, ctypes.c_uint32, ctypes.c_uint32]
        L.oref_synth_mxfp4.restype = None
        L.oref_synth_mxfp4_range.argtypes = [vp, sz, sz, u64, u64, ctypes.c_uint32, ctypes.c_uint32]
        L.oref_synth_mxfp4_range.restype = None
        L.oref_synth_q8_0_range.argtypes = [vp, sz, sz, u64, u64]
        L.oref_synth_q8_0_range.restype = None
        L._synth_bound = True
    return L


def normal_host(n, seed, stream_id, sigma=1.0, mean=0.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    _lib().oref_synth_normal(out.ctypes.data, n, seed, stream_id, sigma, mean)
    return out


def mxfp4_host(blocks, seed, stream_id, scale_lo=SCALE_LO, scale_count=SCALE_COUNT, threads=None) -> np.ndarray:
    """GGUF MXFP4 blocks; large tensors are generated on several host threads
    (the generator is counter-based, so block ranges are independent)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty(blocks * 17, np.uint8)
    L = _lib()
    n = max(1, min(threads or os.cpu_count() or 1, 64, blocks // 65536 + 1))
    cuts = [blocks * i // n for i in range(n + 1)]

    def part(i):
        b0, b1 = cuts[i], cuts[i + 1]
        L.oref_synth_mxfp4_range(out.ctypes.data + 17 * b0, b0, b1 - b0, seed, stream_id, scale_lo, scale_count)

    if n == 1:
        part(0)
    else:
        with ThreadPoolExecutor(n) as ex:
            list(ex.map(part, range(n)))
    return out


def q8_0_host(blocks, seed, stream_id, threads=None) -> np.ndarray:
    """GGUF Q8_0 blocks (34 B: half scale in [2^-11, 2^-9), 32 int8 quants)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    out = np.empty(blocks * 34, np.uint8)
    L = _lib()
    n = max(1, min(threads or os.cpu_count() or 1, 64, blocks // 65536 + 1))
    cuts = [blocks * i // n for i in range(n + 1)]

    def part(i):
        b0, b1 = cuts[i], cuts[i + 1]
        L.oref_synth_q8_0_range(out.ctypes.data + 34 * b0, b0, b1 - b0, seed, stream_id)

    if n == 1:
        part(0)
    else:
        with ThreadPoolExecutor(n) as ex:
            list(ex.map(part, range(n)))
    return out


HEAD_STREAM = 1 << 36


def head_host(seed, rows):
    """The output matrix (Q8_0, rows x 2880) and output_norm.weight ~ N(1, 0.02)."""
    return {"output_w": q8_0_host(rows * (DIM // 32), seed, HEAD_STREAM),
            "output_norm": normal_host(DIM, seed, HEAD_STREAM + 1, 0.02, 1.0)}


def zipf_shift(seed, experts, s, beta=1.0) -> np.ndarray:
    """Router-bias shift beta * ln(p_rank) with p_rank ~ rank^-s; ranks follow a
    seeded permutation so the hot experts are spread over expert ids."""
    draws = normal_host(experts, seed, stream(0, "zipf") + (1 << 20))
    perm = np.argsort(draws, kind="stable")
    rank = np.empty(experts, np.int64)
    rank[perm] = np.arange(1, experts + 1)
    p = rank.astype(np.float64) ** (-s)
    p /= p.sum()
    return (beta * np.log(p)).astype(np.float32)


def layer_host(seed, layer, experts, zipf_s=None, scale_lo=SCALE_LO, scale_count=SCALE_COUNT,
               norm=False) -> dict:
    """One layer's GGUF-layout tensors (numpy)."""
    blocks = experts * DIM * (DIM // 32)
    t = {
        "router_w": normal_host(experts * DIM, seed, stream(layer, "router_w"), 0.02),
        "router_b": normal_host(experts, seed, stream(layer, "router_b"), 0.02),
        "gate_w": mxfp4_host(blocks, seed, stream(layer, "gate_w"), scale_lo, scale_count),
        "gate_b": normal_host(experts * DIM, seed, stream(layer, "gate_b"), 0.02),
        "up_w": mxfp4_host(blocks, seed, stream(layer, "up_w"), scale_lo, scale_count),
        "up_b": normal_host(experts * DIM, seed, stream(layer, "up_b"), 0.02),
        "down_w": mxfp4_host(blocks, seed, stream(layer, "down_w"), scale_lo, scale_count),
        "down_b": normal_host(experts * DIM, seed, stream(layer, "down_b"), 0.02),
    }
    if zipf_s:
        t["router_b"] = (t["router_b"] + zipf_shift(seed, experts, zipf_s)).astype(np.float32)
    if norm:
        t["norm_w"] = normal_host(DIM, seed, stream(layer, "norm_w"), 0.02, 1.0)
    return t


def inputs_host(seed, tokens, batch=0, sigma=1.0) -> np.ndarray:
    """Activations [tokens, 2880] ~ N(0, sigma)."""
    return normal_host(tokens * DIM, seed, INPUT_STREAM_BASE + batch, sigma).reshape(tokens, DIM)
