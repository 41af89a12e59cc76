"""ctypes binding of libttl_moe (include/ttl_moe.h) for Python callers.

The product is the C ABI and the CUDA kernels behind it; this module is the
thin Python mirror that tt-lab-style Python tooling, the tests and bench.py use.
It loads ``tt-lab_b200/lib/libttl_moe.so`` and raises if the library is missing:
there is no Python or CPU fallback for any compute call.

Method names follow tt-lab's model interface: ``moe`` is GptOssModel::moe
(src/model.cpp:292-338), ``moe_batch`` is GptOssModel::moe_batch
(src/model.cpp:340-461), and failures raise RuntimeError with the library's
message, as tt-lab raises std::runtime_error.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

import numpy as np

from . import synth  # noqa: F401  (re-exported helper module)

DIM = 2880
TOPK = 4
BLOCK_BYTES = 17
GGUF_MATRIX_BYTES = DIM * (DIM // 32) * BLOCK_BYTES  # 4,406,400
NCCL_ID_BYTES = 128
TTQ_FORMAT_MXFP4_GPU = 6
TTQ_FORMAT_F32 = 7

TTL_OK = 0
TTL_ERR_ARGUMENT = -1
TTL_ERR_CUDA = -2
TTL_ERR_STATE = -3
TTL_ERR_NCCL = -4
TTL_ERR_DEVICE = -5
TTL_ERR_UNSUPPORTED = -6
TTL_ERR_IO = -7

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = pathlib.Path(os.environ.get("TTL_MOE_LIB", _HERE.parent.parent / "lib" / "libttl_moe.so"))
HEADER_PATH = _HERE.parent.parent.parent / "include" / "ttl_moe.h"


class Config(ctypes.Structure):
    _fields_ = [
        ("experts", ctypes.c_uint32),
        ("layers", ctypes.c_uint32),
        ("max_tokens", ctypes.c_uint32),
        ("device", ctypes.c_int32),
        ("rank", ctypes.c_uint32),
        ("world", ctypes.c_uint32),
        ("nccl_id", ctypes.c_void_p),
        ("flags", ctypes.c_uint32),
    ]


_lib = None


def lib():
    """The loaded libttl_moe (raises OSError when it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise OSError(f"libttl_moe not built: {LIB_PATH} (run `make -C tt-lab_b200`)")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, sz, i32, u32, u64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64
    fp = ctypes.c_void_p
    sig = {
        "ttl_moe_abi_version": (i32, []),
        "ttl_moe_last_error": (ctypes.c_char_p, [vp]),
        "ttl_moe_nccl_id": (i32, [vp]),
        "ttl_moe_create": (i32, [ctypes.POINTER(Config), ctypes.POINTER(vp)]),
        "ttl_moe_destroy": (None, [vp]),
        "ttl_moe_upload_layer": (i32, [vp, i32, fp, fp, vp, fp, vp, fp, vp, fp]),
        "ttl_moe_upload_norm": (i32, [vp, i32, fp]),
        "ttl_moe_upload_layer_packed": (i32, [vp, i32, fp, fp, vp, fp, vp, fp, vp, fp]),
        "ttl_requant_gpu": (i32, [ctypes.c_char_p, ctypes.c_char_p, i32, i32, i32]),
        "ttl_moe_resync": (i32, [vp]),
        "ttl_attn_create": (i32, [vp, ctypes.POINTER(vp)]),
        "ttl_attn_destroy": (None, [vp]),
        "ttl_attn_last_error": (ctypes.c_char_p, [vp]),
        "ttl_attn_upload_layer": (i32, [vp, i32, fp, vp, fp, vp, fp, vp, fp, vp, fp, fp]),
        "ttl_attn_forward_async": (i32, [vp, i32, sz, vp, vp]),
        "ttl_attn_forward": (i32, [vp, i32, sz, vp, vp, vp]),
        "ttl_attn_sync": (i32, [vp]),
        "ttl_attn_stream": (vp, [vp]),
        "ttl_moe_set_timeout": (i32, [vp, u32]),
        "ttl_moe_serve": (i32, [vp, u32]),
        "ttl_moe_decode": (i32, [vp, i32, fp, fp, vp, fp]),
        "ttl_moe_prefill": (i32, [vp, i32, fp, sz, fp, vp, fp]),
        "ttl_moe_forward": (i32, [vp, i32, i32, fp, fp, sz]),
        "ttl_moe_decode_async": (i32, [vp, i32, fp, fp, vp, fp]),
        "ttl_moe_prefill_async": (i32, [vp, i32, fp, sz, fp, vp, fp]),
        "ttl_moe_forward_async": (i32, [vp, i32, i32, fp, fp, sz]),
        "ttl_moe_sync": (i32, [vp]),
        "ttl_moe_stream": (vp, [vp]),
        "ttl_moe_counters": (i32, [vp, ctypes.POINTER(u64), sz]),
        "ttl_moe_profile": (i32, [vp, i32]),
        "ttl_moe_trace": (i32, [vp, i32, ctypes.POINTER(u64)]),
        "ttl_moe_kernel_ms": (i32, [vp, ctypes.POINTER(ctypes.c_float), sz]),
        "ttl_moe_record": (i32, [vp, sz, vp, vp, vp]),
        "ttl_matvec_mxfp4": (i32, [vp, vp, vp, vp, i32]),
        "ttl_matvec_mxfp4_noalloc": (i32, [vp, vp, vp, vp, sz, i32]),
        "ttl_packed_bytes": (sz, [sz]),
        "ttl_pack_mxfp4": (i32, [vp, sz, vp, i32]),
        "ttl_unpack_mxfp4": (i32, [vp, sz, vp, i32]),
        "ttl_ttq_open": (i32, [ctypes.c_char_p, u32, u32, u32, u32, ctypes.POINTER(vp)]),
        "ttl_ttq_add": (i32, [vp, ctypes.c_char_p, u32, u32, ctypes.POINTER(u64), vp, u64]),
        "ttl_ttq_finish": (i32, [vp]),
        "ttl_ttq_close": (None, [vp]),
        "ttl_synth_mxfp4": (i32, [vp, sz, u64, u64, u32, u32]),
        "ttl_synth_normal": (i32, [vp, sz, u64, u64, ctypes.c_float, ctypes.c_float]),
        "ttl_synth_q8_0": (i32, [vp, sz, u64, u64]),
        "ttl_head_create": (i32, [i32, u32, ctypes.POINTER(vp)]),
        "ttl_head_destroy": (None, [vp]),
        "ttl_head_last_error": (ctypes.c_char_p, [vp]),
        "ttl_head_upload": (i32, [vp, vp, fp]),
        "ttl_head_unpack": (i32, [vp, vp]),
        "ttl_head_forward": (i32, [vp, fp, fp, vp]),
        "ttl_head_forward_async": (i32, [vp, fp, fp, vp]),
        "ttl_head_sync": (i32, [vp]),
        "ttl_head_stream": (vp, [vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error(handle=None) -> str:
    msg = lib().ttl_moe_last_error(handle)
    return msg.decode() if msg else ""


def check(rc: int, handle=None):
    if rc != TTL_OK:
        raise RuntimeError(f"cuda moe ({rc}): {last_error(handle)}")


def _ptr(a):
    """Address of a numpy array, a torch tensor, or an int device pointer."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        if not a.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return a.data_ptr()
    raise TypeError(f"unsupported buffer type {type(a)}")


def nccl_id() -> bytes:
    buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
    check(lib().ttl_moe_nccl_id(buf))
    return buf.raw


class MoE:
    """One ttl_moe handle: one GPU, one expert-parallel rank."""

    def __init__(self, experts=32, layers=1, max_tokens=0, device=-1, rank=0, world=1, nccl_id_bytes=None):
        self._id = ctypes.create_string_buffer(nccl_id_bytes, NCCL_ID_BYTES) if nccl_id_bytes else None
        cfg = Config(experts, layers, max_tokens, device, rank, world,
                     ctypes.cast(self._id, ctypes.c_void_p) if self._id is not None else None, 0)
        h = ctypes.c_void_p()
        check(lib().ttl_moe_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h
        self.experts, self.layers, self.max_tokens = experts, layers, max_tokens
        self.rank, self.world = rank, world

    def close(self):
        if getattr(self, "h", None):
            lib().ttl_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc):
        check(rc, self.h)

    def upload_layer(self, layer, t):
        """Binds layer `layer` from a dict of GGUF tensors (host or device)."""
        self._check(lib().ttl_moe_upload_layer(
            self.h, layer, _ptr(t["router_w"]), _ptr(t["router_b"]), _ptr(t["gate_w"]), _ptr(t["gate_b"]),
            _ptr(t["up_w"]), _ptr(t["up_b"]), _ptr(t["down_w"]), _ptr(t["down_b"])))
        if t.get("norm_w") is not None:
            self._check(lib().ttl_moe_upload_norm(self.h, layer, _ptr(t["norm_w"])))

    def upload_layer_packed(self, layer, t):
        """Binds layer `layer` from GPU-layout expert payloads (keys gate_p,
        up_p, down_p: TTQ format-6 bytes of all experts) and the f32 tensors."""
        self._check(lib().ttl_moe_upload_layer_packed(
            self.h, layer, _ptr(t["router_w"]), _ptr(t["router_b"]), _ptr(t["gate_p"]), _ptr(t["gate_b"]),
            _ptr(t["up_p"]), _ptr(t["up_b"]), _ptr(t["down_p"]), _ptr(t["down_b"])))
        if t.get("norm_w") is not None:
            self._check(lib().ttl_moe_upload_norm(self.h, layer, _ptr(t["norm_w"])))

    def moe(self, layer, x):
        """GptOssModel::moe on host f32 [2880]; returns (out, top4 idx, top4 weights)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(DIM, np.float32)
        idx = np.empty(TOPK, np.int32)
        w = np.empty(TOPK, np.float32)
        self._check(lib().ttl_moe_decode(self.h, layer, _ptr(x), _ptr(out), _ptr(idx), _ptr(w)))
        return out, idx, w

    def moe_batch(self, layer, x):
        """GptOssModel::moe_batch on host f32 [T, 2880]; returns (out, idx [T,4], w [T,4])."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, DIM)
        T = x.shape[0]
        out = np.empty((T, DIM), np.float32)
        idx = np.empty((T, TOPK), np.int32)
        w = np.empty((T, TOPK), np.float32)
        self._check(lib().ttl_moe_prefill(self.h, layer, _ptr(x), T, _ptr(out), _ptr(idx), _ptr(w)))
        return out, idx, w

    def forward(self, begin, end, x):
        """RMSNorm -> MoE -> residual through layers [begin, end) for host x [T, 2880]."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, DIM)
        y = np.empty_like(x)
        self._check(lib().ttl_moe_forward(self.h, begin, end, _ptr(x), _ptr(y), x.shape[0]))
        return y

    def decode_async(self, layer, x, out, idx=None, w=None):
        self._check(lib().ttl_moe_decode_async(self.h, layer, _ptr(x), _ptr(out), _ptr(idx), _ptr(w)))

    def prefill_async(self, layer, x, tokens, out, idx=None, w=None):
        self._check(lib().ttl_moe_prefill_async(self.h, layer, _ptr(x), tokens, _ptr(out), _ptr(idx), _ptr(w)))

    def forward_async(self, begin, end, x, y, tokens):
        self._check(lib().ttl_moe_forward_async(self.h, begin, end, _ptr(x), _ptr(y), tokens))

    def prefill_host(self, layer, x, tokens, out, idx=None, w=None):
        """ttl_moe_prefill on caller-owned host buffers (pinned or pageable)."""
        self._check(lib().ttl_moe_prefill(self.h, layer, _ptr(x), tokens, _ptr(out), _ptr(idx), _ptr(w)))

    def forward_host(self, begin, end, x, y, tokens):
        """ttl_moe_forward on caller-owned host buffers (pinned or pageable)."""
        self._check(lib().ttl_moe_forward(self.h, begin, end, _ptr(x), _ptr(y), tokens))

    def sync(self):
        self._check(lib().ttl_moe_sync(self.h))

    def resync(self):
        """Collective: brings the ranks back into agreement after a failed call."""
        self._check(lib().ttl_moe_resync(self.h))

    def set_timeout(self, ms):
        self._check(lib().ttl_moe_set_timeout(self.h, int(ms)))

    def serve(self, idle_us):
        """Blocking decode calls through a resident decode kernel (0: off)."""
        self._check(lib().ttl_moe_serve(self.h, int(idle_us)))

    def stream(self) -> int:
        return lib().ttl_moe_stream(self.h) or 0

    def profile(self, enable=True):
        self._check(lib().ttl_moe_profile(self.h, 1 if enable else 0))

    def kernel_ms(self):
        """Duration of the last profiled decode-kernel launch: (ms, steps, persistent)."""
        out = (ctypes.c_float * 3)()
        self._check(lib().ttl_moe_kernel_ms(self.h, out, 3))
        return {"ms": out[0], "steps": int(out[1]), "persistent": bool(out[2])}

    def trace_enable(self, steps):
        self._check(lib().ttl_moe_trace(self.h, steps, None))
        self._trace_steps = steps

    def trace(self):
        """[steps, 10] ns stamps of the persistent decode kernel's phases."""
        n = self._trace_steps
        out = (ctypes.c_uint64 * (n * 10))()
        self._check(lib().ttl_moe_trace(self.h, 0, out))
        return np.frombuffer(out, dtype=np.uint64).reshape(n, 10).astype(np.int64)

    def record(self, steps, y_log=None, idx_log=None, w_log=None):
        """Step log of later forward/decode launches into caller-owned device
        buffers (y_log [steps, 2880] f32, idx_log / w_log [steps, 4]);
        steps = 0 turns it off."""
        self._check(lib().ttl_moe_record(self.h, steps, _ptr(y_log), _ptr(idx_log), _ptr(w_log)))

    def counters(self):
        out = (ctypes.c_uint64 * 4)()
        n = lib().ttl_moe_counters(self.h, out, 4)
        vals = [int(out[i]) for i in range(n)]
        return {"router_exact_reevals": vals[0], "prefill_reevals": vals[1], "launches": vals[2],
                "persistent_decode": vals[3]}


def packed_bytes(matrices: int) -> int:
    return lib().ttl_packed_bytes(matrices)


def pack_mxfp4(gguf, matrices, packed=None, device=0):
    if packed is None:
        packed = np.empty(packed_bytes(matrices), np.uint8)
    check(lib().ttl_pack_mxfp4(_ptr(gguf), matrices, _ptr(packed), device))
    return packed


def requant_gpu(gguf_path, ttq_path, layer_begin=0, layer_end=-1, device=0):
    """requant --cuda: a gpt-oss GGUF to a TTQ file with GPU-layout experts."""
    check(lib().ttl_requant_gpu(str(gguf_path).encode(), str(ttq_path).encode(), layer_begin, layer_end, device))


def matvec_mxfp4(packed, bias, x, y, device=0):
    """y = bias + W x on the tensor cores (device tensors)."""
    check(lib().ttl_matvec_mxfp4(_ptr(packed), _ptr(bias), _ptr(x), _ptr(y), device))
    return y


def matvec_mxfp4_noalloc(packed, bias, x, y, matrices=1, device=0):
    """matvec_mxfp4 over `matrices` consecutive problems without allocating
    device memory (at most 256 per call)."""
    check(lib().ttl_matvec_mxfp4_noalloc(_ptr(packed), _ptr(bias), _ptr(x), _ptr(y), matrices, device))
    return y


def unpack_mxfp4(packed, matrices, gguf=None, device=0):
    if gguf is None:
        gguf = np.empty(matrices * GGUF_MATRIX_BYTES, np.uint8)
    check(lib().ttl_unpack_mxfp4(_ptr(packed), matrices, _ptr(gguf), device))
    return gguf


class Head:
    """One ttl_head handle: the output head of GptOssModel::forward (rms_norm
    with output_norm.weight, matvec_q8_0 with output.weight, greedy)."""

    def __init__(self, vocab=201088, device=-1):
        h = ctypes.c_void_p()
        check(lib().ttl_head_create(device, vocab, ctypes.byref(h)))
        self.h = h
        self.vocab = vocab

    def _check(self, rc):
        if rc != TTL_OK:
            msg = lib().ttl_head_last_error(self.h)
            raise RuntimeError(f"cuda head ({rc}): {msg.decode() if msg else ''}")

    def close(self):
        if getattr(self, "h", None):
            lib().ttl_head_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def upload(self, q8_0, norm_w):
        self._check(lib().ttl_head_upload(self.h, _ptr(q8_0), _ptr(norm_w)))

    def unpack(self):
        out = np.empty(self.vocab * (DIM // 32) * 34, np.uint8)
        self._check(lib().ttl_head_unpack(self.h, _ptr(out)))
        return out

    def forward(self, x, want_logits=True):
        """Host x [2880] -> (logits [vocab] or None, token)."""
        x = np.ascontiguousarray(x, np.float32)
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        tok = np.zeros(1, np.int32)
        self._check(lib().ttl_head_forward(self.h, _ptr(x), _ptr(logits), _ptr(tok)))
        return logits, int(tok[0])

    def forward_async(self, x, logits=None, token=None):
        self._check(lib().ttl_head_forward_async(self.h, _ptr(x), _ptr(logits), _ptr(token)))

    def sync(self):
        self._check(lib().ttl_head_sync(self.h))

    def stream(self) -> int:
        return lib().ttl_head_stream(self.h) or 0


class AttnConfig(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_uint32), ("token_capacity", ctypes.c_uint32), ("device", ctypes.c_int32),
                ("stream", ctypes.c_void_p)]


class Attention:
    """One ttl_attn handle: the attention block of GptOssModel::forward
    (rms_norm, Q/K/V Q8_0 projections, RoPE, KV cache, attention with sinks,
    output projection, residual) for `layers` layers."""

    def __init__(self, layers=1, token_capacity=256, device=-1, stream=None):
        cfg = AttnConfig(layers, token_capacity, device, stream)
        h = ctypes.c_void_p()
        check(lib().ttl_attn_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h

    def _check(self, rc):
        if rc != TTL_OK:
            msg = lib().ttl_attn_last_error(self.h)
            raise RuntimeError(f"cuda attention ({rc}): {msg.decode() if msg else ''}")

    def close(self):
        if getattr(self, "h", None):
            lib().ttl_attn_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def upload_layer(self, layer, t):
        self._check(lib().ttl_attn_upload_layer(
            self.h, layer, _ptr(t["attn_norm"]), _ptr(t["q_w"]), _ptr(t["q_b"]), _ptr(t["k_w"]), _ptr(t["k_b"]),
            _ptr(t["v_w"]), _ptr(t["v_b"]), _ptr(t["o_w"]), _ptr(t["o_b"]), _ptr(t["sinks"])))

    def forward(self, layer, position, x):
        """Host x [2880] -> (residual [2880], attended [4096])."""
        x = np.ascontiguousarray(x, np.float32)
        res = np.empty(DIM, np.float32)
        att = np.empty(4096, np.float32)
        self._check(lib().ttl_attn_forward(self.h, layer, position, _ptr(x), _ptr(res), _ptr(att)))
        return res, att

    def forward_async(self, layer, position, x, residual):
        self._check(lib().ttl_attn_forward_async(self.h, layer, position, _ptr(x), _ptr(residual)))

    def sync(self):
        self._check(lib().ttl_attn_sync(self.h))

    def stream(self) -> int:
        return lib().ttl_attn_stream(self.h) or 0


class TtqWriter:
    """Atomic TTLBQNT1 writer (tt-lab src/requant.cpp:23-68, :415-504)."""

    def __init__(self, path, model, layers, experts, tensor_count):
        w = ctypes.c_void_p()
        check(lib().ttl_ttq_open(str(path).encode(), model, layers, experts, tensor_count, ctypes.byref(w)))
        self.w = w

    def add(self, name, fmt, shape, payload):
        payload = np.ascontiguousarray(payload)
        shp = (ctypes.c_uint64 * 4)(*([int(s) for s in shape] + [0] * (4 - len(shape))))
        check(lib().ttl_ttq_add(self.w, name.encode(), fmt, len(shape), shp, _ptr(payload), payload.nbytes))

    def finish(self):
        check(lib().ttl_ttq_finish(self.w))

    def close(self):
        if self.w:
            lib().ttl_ttq_close(self.w)
            self.w = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
