"""A minimal GGUF v3 writer for tests: metadata and tensors of a gpt-oss
MoE model, laid out as the format defines it (header, key/values, tensor
directory, aligned data) -- what tt-lab's reader parses (src/gguf.cpp)."""
import struct

import numpy as np

F32, MXFP4 = 0, 39
U32, STRING = 4, 8


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def gpt_oss_meta(model_layers=24, experts=32, architecture="gpt-oss"):
    return [("general.architecture", STRING, architecture), ("gpt-oss.block_count", U32, model_layers),
            ("gpt-oss.expert_count", U32, experts), ("gpt-oss.embedding_length", U32, 2880),
            ("general.alignment", U32, 32)]


def moe_tensors(layer, t, experts=32):
    """(name, type, GGUF shape (innermost first), array) of one layer's MoE
    tensors from a synthetic-layer dict."""
    p = f"blk.{layer}."
    out = [(p + "ffn_gate_inp.weight", F32, [2880, experts], t["router_w"]),
           (p + "ffn_gate_inp.bias", F32, [experts], t["router_b"])]
    for m in ("gate", "up", "down"):
        out += [(p + f"ffn_{m}_exps.weight", MXFP4, [2880, 2880, experts], t[f"{m}_w"]),
                (p + f"ffn_{m}_exps.bias", F32, [2880, experts], t[f"{m}_b"])]
    return out


def write_gguf(path, meta, tensors):
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, typ, v in meta:
        head += _str(k) + struct.pack("<I", typ) + (_str(v) if typ == STRING else struct.pack("<I", v))
    offsets, off = [], 0
    for name, typ, shape, arr in tensors:
        off = (off + 31) // 32 * 32
        offsets.append(off)
        off += np.asarray(arr).nbytes
    for (name, typ, shape, arr), o in zip(tensors, offsets):
        head += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", typ, o)
    base = (len(head) + 31) // 32 * 32
    with open(path, "wb") as f:
        f.write(head + b"\0" * (base - len(head)))
        for (name, typ, shape, arr), o in zip(tensors, offsets):
            f.seek(base + o)
            f.write(np.ascontiguousarray(arr).tobytes())
