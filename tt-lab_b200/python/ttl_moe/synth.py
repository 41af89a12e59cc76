"""Seeded synthetic gpt-oss MoE layers and activations (the benchmark configs).

No gpt-oss GGUF is available to the tests or the benchmark, so every tensor is
generated from (seed, stream) by the library's counter-based generator
(csrc/synth.h), identically on host and device:

  router W [E][2880] ~ N(0, 0.02), router bias ~ N(0, 0.02) (+ optional Zipf shift)
  expert W  MXFP4 GGUF blocks: nibbles uniform over the 16 E2M1 codes, E8M0 scale
            bytes uniform over 119..125 (unbiased exponent -8..-2)
  expert biases ~ N(0, 0.02); activations ~ N(0, 1)

"N(0, s)" is s * (sum of twelve 24-bit uniforms - 6) (Irwin-Hall), which has
mean 0 and variance s^2 and is computed in integers so host and device agree.
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


def stream(layer: int, name: str) -> int:
    return layer * 16 + _KINDS[name]


def _lib():
    from . import lib
    return lib()


def _check(rc):
    from . import check
    check(rc)


def normal_host(n, seed, stream_id, sigma=1.0, mean=0.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(_lib().ttl_synth_normal(out.ctypes.data, n, seed, stream_id, ctypes.c_float(sigma), ctypes.c_float(mean)))
    return out


def mxfp4_host(blocks, seed, stream_id, scale_lo=SCALE_LO, scale_count=SCALE_COUNT) -> np.ndarray:
    out = np.empty(blocks * 17, np.uint8)
    _check(_lib().ttl_synth_mxfp4(out.ctypes.data, blocks, seed, stream_id, scale_lo, scale_count))
    return out


def zipf_shift(seed, experts, s, beta=1.0) -> np.ndarray:
    """Router-bias shift beta * ln(p_rank) with p_rank ~ rank^-s; ranks follow a
    seeded permutation so the hot experts are spread over expert ids."""
    draws = normal_host(experts, seed, stream(0, "zipf") + (1 << 20))
    perm = np.argsort(draws, kind="stable")  # perm[r] = expert of rank r+1
    rank = np.empty(experts, np.int64)
    rank[perm] = np.arange(1, experts + 1)
    p = rank.astype(np.float64) ** (-s)
    p /= p.sum()
    return (beta * np.log(p)).astype(np.float32)


def layer_host(seed, layer, experts, zipf_s=None, scale_lo=SCALE_LO, scale_count=SCALE_COUNT,
               norm=False) -> dict:
    """One layer's GGUF-layout tensors on the host (numpy)."""
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


def layer_device(seed, layer, experts, device="cuda", zipf_s=None, scale_lo=SCALE_LO, scale_count=SCALE_COUNT):
    """The same tensors as layer_host, generated directly in device memory
    (torch tensors) -- used for multi-GB stacks."""
    import torch
    blocks = experts * DIM * (DIM // 32)
    t = {}
    for name, sigma in (("router_w", 0.02), ("router_b", 0.02), ("gate_b", 0.02), ("up_b", 0.02), ("down_b", 0.02)):
        n = experts * DIM if name != "router_b" else experts
        buf = torch.empty(n, dtype=torch.float32, device=device)
        _check(_lib().ttl_synth_normal(buf.data_ptr(), n, seed, stream(layer, name), ctypes.c_float(sigma),
                                       ctypes.c_float(0.0)))
        t[name] = buf
    for name in ("gate_w", "up_w", "down_w"):
        buf = torch.empty(blocks * 17, dtype=torch.uint8, device=device)
        _check(_lib().ttl_synth_mxfp4(buf.data_ptr(), blocks, seed, stream(layer, name), scale_lo, scale_count))
        t[name] = buf
    if zipf_s:
        t["router_b"] += torch.from_numpy(zipf_shift(seed, experts, zipf_s)).to(device)
    return t


HEAD_STREAM = 1 << 36


def head_device(seed, rows, device="cuda"):
    """The output matrix (Q8_0, rows x 2880) and output_norm.weight ~ N(1,
    0.02) in device memory (torch tensors)."""
    import torch
    w = torch.empty(rows * (DIM // 32) * 34, dtype=torch.uint8, device=device)
    _check(_lib().ttl_synth_q8_0(w.data_ptr(), rows * (DIM // 32), seed, HEAD_STREAM))
    g = torch.empty(DIM, dtype=torch.float32, device=device)
    _check(_lib().ttl_synth_normal(g.data_ptr(), DIM, seed, HEAD_STREAM + 1, ctypes.c_float(0.02), ctypes.c_float(1.0)))
    return {"output_w": w, "output_norm": g}


def q8_0_host(blocks, seed, stream_id) -> np.ndarray:
    out = np.empty(blocks * 34, np.uint8)
    _check(_lib().ttl_synth_q8_0(out.ctypes.data, blocks, seed, stream_id))
    return out


def inputs_host(seed, tokens, batch=0, sigma=1.0) -> np.ndarray:
    """Activations [tokens, 2880] ~ N(0, sigma)."""
    return normal_host(tokens * DIM, seed, INPUT_STREAM_BASE + batch, sigma).reshape(tokens, DIM)


ATTN_STREAM = 1 << 37
_ATTN_KINDS = {"attn_norm": 0, "q_w": 1, "q_b": 2, "k_w": 3, "k_b": 4, "v_w": 5, "v_b": 6, "o_w": 7, "o_b": 8,
               "sinks": 9}


def attention_layer_host(seed, layer) -> dict:
    """One layer's attention tensors in GGUF layout (numpy): attn_norm ~
    N(1, 0.02); Q8_0 Q [4096 x 2880], K, V [512 x 2880], O [2880 x 4096]
    (the generator's Q8_0 blocks; the Q and K block scales divided by 4 so
    that scores q.k / 8 stay of order 1); biases ~ N(0, 0.02); sinks ~ N(0, 1)."""
    st = lambda k: ATTN_STREAM + layer * 16 + _ATTN_KINDS[k]  # noqa: E731
    t = {"attn_norm": normal_host(DIM, seed, st("attn_norm"), 0.02, 1.0)}
    for name, rows, cols in (("q_w", 4096, DIM), ("k_w", 512, DIM), ("v_w", 512, DIM), ("o_w", DIM, 4096)):
        w = q8_0_host(rows * cols // 32, seed, st(name))
        if name in ("q_w", "k_w"):
            blk = w.reshape(-1, 34)
            bits = blk[:, 0].astype(np.uint16) | (blk[:, 1].astype(np.uint16) << 8)
            bits = bits - np.uint16(0x0800)  # fp16 exponent - 2: the scale / 4
            blk[:, 0] = (bits & 0xFF).astype(np.uint8)
            blk[:, 1] = (bits >> 8).astype(np.uint8)
        t[name] = w
    for name, n in (("q_b", 4096), ("k_b", 512), ("v_b", 512), ("o_b", DIM)):
        t[name] = normal_host(n, seed, st(name), 0.02)
    t["sinks"] = normal_host(64, seed, st("sinks"), 1.0)
    return t
