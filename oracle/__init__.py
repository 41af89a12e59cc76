"""CPU oracle for the gpt-oss MoE path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs use this package, and only as the checker; the product (libttl_moe) never
links or calls it.

Two oracles, both built by oracle/Makefile:
  * ``port``      -- oracle/moe_oracle.c, a plain-C restatement of tt-lab's
                     algorithm with each function citing the reference file:line;
  * ``reference`` -- oracle/_ref/libttlref.so, tt-lab's own src/tensor.cpp,
                     src/gguf.cpp and src/model.cpp compiled unmodified, driven
                     through ref_shim.cpp (GptOssModel::moe / moe_batch).
The port is pinned against the reference's known-answer vectors and against the
compiled reference bit for bit (tests/test_oracle.py).
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
PORT_PATH = HERE / "_build" / "libmoe_oracle.so"
REF_PATH = HERE / "_ref" / "libttlref.so"
DIM = 2880
ISA_DEFAULT = 0
ISA_V4 = 1

_port = None
_ref = None


class _Layer(ctypes.Structure):
    _fields_ = [("experts", ctypes.c_size_t)] + [
        (n, ctypes.c_void_p) for n in ("router_w", "router_b", "gate_w", "up_w", "down_w", "gate_b", "up_b",
                                        "down_b")]


def _p(a):
    return None if a is None else a.ctypes.data


def port():
    global _port
    if _port is None:
        if not PORT_PATH.exists():
            raise OSError(f"oracle not built: {PORT_PATH} (make -C oracle oracle)")
        L = ctypes.CDLL(str(PORT_PATH))
        vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        L.oref_mxfp4_scale.restype = ctypes.c_float
        L.oref_mxfp4_scale.argtypes = [ctypes.c_uint8]
        L.oref_matvec_add_mxfp4.argtypes = [vp, vp, vp, vp, i32]
        L.oref_matmul_add_mxfp4_selected.argtypes = [vp, vp, vp, vp, sz, vp, i32]
        L.oref_moe_decode.argtypes = [ctypes.POINTER(_Layer), vp, vp, vp, vp, i32]
        L.oref_moe_prefill.argtypes = [ctypes.POINTER(_Layer), vp, sz, vp, vp, vp, i32]
        L.oref_moe_prefill.restype = i32
        L.oref_rms_norm.argtypes = [vp, vp, ctypes.c_float, vp, sz]
        L.oref_select_top4.argtypes = [vp, sz, vp]
        L.oref_softmax4.argtypes = [vp, vp, vp]
        L.oref_swiglu.restype = ctypes.c_float
        L.oref_swiglu.argtypes = [ctypes.c_float, ctypes.c_float]
        L.oref_matvec_add_f32.argtypes = [vp, vp, vp, vp, sz, sz]
        L.oref_matvec_q8_0.argtypes = [vp, vp, vp, sz]
        L.oref_greedy.argtypes = [vp, sz]
        L.oref_greedy.restype = ctypes.c_int32
        L.oref_half_to_float.argtypes = [ctypes.c_uint16]
        L.oref_half_to_float.restype = ctypes.c_float
        L.oref_attention_step.argtypes = [ctypes.POINTER(_AttnLayer), sz, sz, vp, vp, sz, vp, vp, vp]
        L.oref_attention_step.restype = i32
        L.oref_rope_frequencies.argtypes = [vp]
        _port = L
    return _port


def ref_available() -> bool:
    return REF_PATH.exists()


def ref():
    global _ref
    if _ref is None:
        if not REF_PATH.exists():
            raise OSError(f"reference oracle not built: {REF_PATH} (make -C oracle ref)")
        L = ctypes.CDLL(str(REF_PATH))
        vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        L.tref_last_error.restype = ctypes.c_char_p
        L.tref_isa_v4.restype = i32
        L.tref_mxfp4_scale.restype = ctypes.c_float
        L.tref_mxfp4_scale.argtypes = [ctypes.c_uint8]
        L.tref_matvec_add_mxfp4.argtypes = [vp, vp, sz, sz, vp, vp, i32]
        L.tref_matmul_add_mxfp4_selected.argtypes = [vp, vp, sz, sz, vp, vp, sz, vp, i32]
        L.tref_rms_norm.argtypes = [vp, vp, ctypes.c_float, vp, sz]
        L.tref_moe_decode.argtypes = [sz] + [vp] * 12
        L.tref_moe_prefill.argtypes = [sz] + [vp] * 9 + [sz, vp, vp, vp]
        L.tref_moe_decode_threaded.argtypes = [sz] + [vp] * 10 + [i32]
        L.tref_moe_layer_tokens.argtypes = [sz, vp, vp, vp, vp, sz, i32, vp, vp, vp]
        L.tref_forward_tokens.argtypes = [sz, sz, vp, vp, vp, vp, sz, i32]
        L.tref_matvec_q8_0.argtypes = [vp, sz, vp, vp, vp]
        L.tref_greedy.argtypes = [vp, vp]
        L.tref_attention_steps.argtypes = [ctypes.POINTER(vp), i32, sz, vp, vp, vp]
        _ref = L
    return _ref


class _AttnLayer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("attn_norm", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b",
                                               "sinks")]


ATTN_TENSORS = ("attn_norm", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "sinks")


def attention_steps(t, layer_index, x, impl="port"):
    """The attention block of GptOssModel::forward (src/model.cpp:578-590)
    for positions 0 .. P-1 of one layer (even index: sliding window), x
    [P][2880] one row per position.  Returns (residual [P][2880], attended
    [P][4096]).  impl "port": the C restatement (attn_oracle.c); "ref": tt-lab's
    own code (tref_attention_steps)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, DIM)
    P = x.shape[0]
    res = np.empty((P, DIM), np.float32)
    att = np.empty((P, 4096), np.float32)
    if impl == "ref":
        ptrs = (ctypes.c_void_p * 10)(*[t[n].ctypes.data for n in ATTN_TENSORS])
        _ref_check(ref().tref_attention_steps(ptrs, layer_index, P, _p(x), _p(res), _p(att)))
        return res, att
    L = _AttnLayer(*[t[n].ctypes.data for n in ATTN_TENSORS])
    kc = np.zeros((P, 512), np.float32)
    vc = np.zeros((P, 512), np.float32)
    for p in range(P):
        rc = port().oref_attention_step(ctypes.byref(L), layer_index, p, _p(kc), _p(vc), P, _p(x[p]), _p(res[p]),
                                        _p(att[p]))
        if rc != 0:
            raise RuntimeError("oref_attention_step failed")
    return res, att


def rope_frequencies():
    f = np.empty(32, np.float32)
    port().oref_rope_frequencies(_p(f))
    return f


def _ref_check(rc):
    if rc != 0:
        raise RuntimeError("reference oracle: " + (ref().tref_last_error() or b"").decode())


def _layer(t):
    experts = t["router_b"].shape[0]
    return _Layer(experts, *[t[n].ctypes.data for n in ("router_w", "router_b", "gate_w", "up_w", "down_w",
                                                          "gate_b", "up_b", "down_b")])


def moe_decode(t, x, isa=ISA_V4, impl="port"):
    """Decode MoE of one token.  Returns (out [2880], idx [4], w [4])."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(DIM, np.float32)
    idx = np.empty(4, np.int32)
    w = np.empty(4, np.float32)
    if impl == "port":
        lay = _layer(t)
        port().oref_moe_decode(ctypes.byref(lay), _p(x), _p(out), _p(idx), _p(w), isa)
    else:
        _ref_check(ref().tref_moe_decode(t["router_b"].shape[0], _p(t["router_w"]), _p(t["router_b"]),
                                         _p(t["gate_w"]), _p(t["gate_b"]), _p(t["up_w"]), _p(t["up_b"]),
                                         _p(t["down_w"]), _p(t["down_b"]), _p(x), _p(out), _p(idx), _p(w)))
    return out, idx, w


def moe_prefill(t, x, isa=ISA_V4, impl="port"):
    """Prefill MoE of x [T, 2880].  Returns (out [T,2880], idx [T,4], w [T,4])."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, DIM)
    T = x.shape[0]
    out = np.empty((T, DIM), np.float32)
    idx = np.empty((T, 4), np.int32)
    w = np.empty((T, 4), np.float32)
    if impl == "port":
        lay = _layer(t)
        if port().oref_moe_prefill(ctypes.byref(lay), _p(x), T, _p(out), _p(idx), _p(w), isa) != 0:
            raise MemoryError("oracle prefill allocation failed")
    else:
        _ref_check(ref().tref_moe_prefill(t["router_b"].shape[0], _p(t["router_w"]), _p(t["router_b"]),
                                          _p(t["gate_w"]), _p(t["gate_b"]), _p(t["up_w"]), _p(t["up_b"]),
                                          _p(t["down_w"]), _p(t["down_b"]), _p(x), T, _p(out), _p(idx), _p(w)))
    return out, idx, w


VOCAB = 201088


def matvec_q8_0(w, x, rows, impl="port"):
    """tt-lab's matvec_q8_0 (src/tensor.cpp:202-218) of `rows` GGUF Q8_0 rows
    (uint8 [rows * 3060]) with x [2880].  Returns f32 [rows]."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(rows, np.float32)
    if impl == "port":
        port().oref_matvec_q8_0(_p(w), _p(x), _p(y), rows)
    else:
        _ref_check(ref().tref_matvec_q8_0(_p(w), rows, _p(x), _p(y), None))
    return y


def greedy(logits, impl="port"):
    """GptOssModel::greedy (src/model.cpp:604-612)."""
    logits = np.ascontiguousarray(logits, np.float32)
    if impl == "port":
        return int(port().oref_greedy(_p(logits), logits.size))
    if logits.size != VOCAB:
        raise ValueError("the reference's greedy reads the full vocabulary")
    tok = np.zeros(1, np.int32)
    _ref_check(ref().tref_greedy(_p(logits), _p(tok)))
    return int(tok[0])


def head(w, norm_w, x, rows, impl="port"):
    """The output head of GptOssModel::forward (src/model.cpp:598-612):
    rms_norm(x, norm_w) -> matvec_q8_0 -> greedy.  Returns (logits, token)."""
    h = rms_norm(x, norm_w, impl=impl)
    logits = matvec_q8_0(w, h, rows, impl=impl)
    return logits, greedy(logits, impl="port" if rows != VOCAB else impl)


def router_logits(t, x):
    """tt-lab's router chain for each row of x (matvec_add_f32,
    src/tensor.cpp:186-200: bias first, products rounded, added in column
    order; the prefill's matmul_add_f32 keeps the same per-token order).
    Returns [T, E]."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, DIM)
    E = t["router_b"].shape[0]
    out = np.empty((x.shape[0], E), np.float32)
    for i in range(x.shape[0]):
        port().oref_matvec_add_f32(_p(t["router_w"]), _p(t["router_b"]), _p(x[i]), _p(out[i]), E, DIM)
    return out


def rms_norm(x, g, eps=1.0e-5, impl="port"):
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty_like(x)
    if impl == "port":
        port().oref_rms_norm(_p(x), _p(g), ctypes.c_float(eps), _p(out), x.size)
    else:
        _ref_check(ref().tref_rms_norm(_p(x), _p(g), ctypes.c_float(eps), _p(out), x.size))
    return out


def forward(layers, x, isa=ISA_V4, impl="port"):
    """Per token: for each layer h = rms_norm(x, norm_w); x = x + moe(h)
    (tt-lab src/model.cpp:590-594).  layers: list of tensor dicts."""
    x = np.array(x, np.float32).reshape(-1, DIM)
    ones = np.ones(DIM, np.float32)
    for t in range(x.shape[0]):
        cur = x[t].copy()
        for lay in layers:
            h = rms_norm(cur, lay.get("norm_w", ones), impl=impl)
            out, _, _ = moe_decode(lay, h, isa, impl)
            cur = (cur + out).astype(np.float32)
        x[t] = cur
    return x


_TENSORS = ("router_w", "router_b", "gate_w", "gate_b", "up_w", "up_b", "down_w", "down_b")


def _table(layers):
    """Pointer table for the reference drivers: 8 tensor pointers per layer
    (router_w, router_b, gate_w, gate_b, up_w, up_b, down_w, down_b)."""
    arr = (ctypes.c_void_p * (8 * len(layers)))()
    for l, t in enumerate(layers):
        for k, n in enumerate(_TENSORS):
            a = t[n]
            if not (a.flags["C_CONTIGUOUS"] and a.dtype in (np.float32, np.uint8)):
                raise ValueError(f"layer {l} tensor {n} must be contiguous f32 / u8")
            arr[8 * l + k] = a.ctypes.data
    return arr


def moe_layer_tokens(t, x, norm_w=None, threads=None):
    """One layer for many independent tokens through tt-lab's own code
    (rms_norm + GptOssModel::moe + residual, src/model.cpp:590-594), on host
    threads.  Returns (y [T,2880], idx [T,4], w [T,4], router logits [T,E])."""
    import os
    x = np.ascontiguousarray(x, np.float32).reshape(-1, DIM)
    T = x.shape[0]
    E = t["router_b"].shape[0]
    y = np.empty_like(x)
    idx = np.empty((T, 4), np.int32)
    w = np.empty((T, 4), np.float32)
    logits = np.empty((T, E), np.float32)
    g = None if norm_w is None else np.ascontiguousarray(norm_w, np.float32)
    tab = _table([t])
    n = threads or os.cpu_count() or 1
    _ref_check(ref().tref_moe_layer_tokens(E, tab, _p(g), _p(x), _p(y), T, int(n), _p(idx), _p(w), _p(logits)))
    return y, idx, w, logits


def forward_tokens(layers, x, threads=None, norms=None):
    """Token-major decode of independent tokens through all `layers` with
    tt-lab's own code (one worker per host thread, each token as
    GptOssModel::forward runs it, attention left out).  Returns y [T,2880]."""
    import os
    x = np.ascontiguousarray(x, np.float32).reshape(-1, DIM)
    T = x.shape[0]
    E = layers[0]["router_b"].shape[0]
    y = np.empty_like(x)
    tab = _table(layers)
    nptr = None
    if norms is not None:
        nptr = (ctypes.c_void_p * len(layers))(*[None if g is None else g.ctypes.data for g in norms])
    n = threads or os.cpu_count() or 1
    _ref_check(ref().tref_forward_tokens(E, len(layers), tab, nptr, _p(x), _p(y), T, int(n)))
    return y


def compare(a, b):
    """tt-lab's compare_vectors metrics (src/tt_backend.cpp:3100-3128) plus the
    max error relative to max |b| used as the parity bar."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    err = a - b
    rms_b = np.sqrt(np.mean(b * b))
    return {
        "max_abs": float(np.max(np.abs(err))),
        "max_rel": float(np.max(np.abs(err)) / max(np.max(np.abs(b)), 1e-30)),
        "rel_rms": float(np.sqrt(np.mean(err * err)) / max(rms_b, 1e-30)),
        "cosine": float(np.dot(a, b) / max(np.sqrt(np.dot(a, a) * np.dot(b, b)), 1e-30)),
    }


# ---- tt-lab's TTQ reader (TtqFile, src/tt_backend.cpp:315-445) ----
TTQ_PATH = HERE / "_ref" / "libttlttq.so"
_ttq = None


def ttq_available() -> bool:
    return TTQ_PATH.exists()


def _ttq_lib():
    global _ttq
    if _ttq is None:
        if not TTQ_PATH.exists():
            raise OSError(f"TTQ reader not built: {TTQ_PATH} (make -C oracle ttq)")
        L = ctypes.CDLL(str(TTQ_PATH))
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        L.tref_ttq_last_error.restype = ctypes.c_char_p
        L.tref_ttq_open.restype = vp
        L.tref_ttq_open.argtypes = [ctypes.c_char_p]
        L.tref_ttq_close.argtypes = [vp]
        L.tref_ttq_count.restype = sz
        L.tref_ttq_count.argtypes = [vp]
        L.tref_ttq_layers.restype = sz
        L.tref_ttq_layers.argtypes = [vp]
        L.tref_ttq_record.argtypes = [vp, sz, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32),
                                      ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64)]
        _ttq = L
    return _ttq


def ttq_read(path):
    """Every record of a TTQ file as tt-lab's TtqFile parses it: a list of
    dicts (name, format, shape, payload as a read-only numpy view).  The file
    stays mapped while the returned object lives."""
    L = _ttq_lib()
    f = L.tref_ttq_open(str(path).encode())
    if not f:
        raise RuntimeError("TtqFile: " + L.tref_ttq_last_error().decode())

    class Mapped(list):
        def __del__(self):
            L.tref_ttq_close(f)

    out = Mapped()
    out.layers = int(L.tref_ttq_layers(f))
    name = ctypes.create_string_buffer(128)
    fmt, rank = ctypes.c_uint32(), ctypes.c_uint32()
    shape = (ctypes.c_uint64 * 4)()
    data, size = ctypes.c_void_p(), ctypes.c_uint64()
    for i in range(int(L.tref_ttq_count(f))):
        L.tref_ttq_record(f, i, name, ctypes.byref(fmt), ctypes.byref(rank), shape, ctypes.byref(data),
                          ctypes.byref(size))
        buf = (ctypes.c_uint8 * size.value).from_address(data.value) if size.value else (ctypes.c_uint8 * 0)()
        out.append({"name": name.value.decode(), "format": fmt.value,
                    "shape": [int(shape[d]) for d in range(rank.value)],
                    "payload": np.frombuffer(buf, np.uint8)})
    return out
