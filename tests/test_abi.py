"""Host-side checks of the C ABI (no GPU needed): every symbol declared in
include/ttl_moe.h is exported, argument validation and the no-device error,
the TTQ container writer (tt-lab src/requant.cpp:23-68, :415-504) and the
C++ wrapper header."""
import os
import pathlib
import re
import struct
import subprocess

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ttl_moe.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ttl_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    import ttl_moe
    L = ttl_moe.lib()
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert L.ttl_moe_abi_version() == 1


def test_binding_covers_header():
    import ttl_moe
    src = (ROOT / "tt-lab_b200" / "python" / "ttl_moe" / "__init__.py").read_text()
    for n in declared_functions():
        assert f'"{n}"' in src, n


def test_create_validates_config():
    import ttl_moe
    with pytest.raises(RuntimeError, match="experts must be 32 or 128"):
        ttl_moe.MoE(experts=16)
    with pytest.raises(RuntimeError, match="world must be"):
        ttl_moe.MoE(experts=32, world=3)
    with pytest.raises(RuntimeError, match="NCCL id"):
        ttl_moe.MoE(experts=32, world=2, rank=1)


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="a GPU is present")
def test_create_without_gpu_fails_loudly():
    import ttl_moe
    with pytest.raises(RuntimeError, match="no CUDA device"):
        ttl_moe.MoE(experts=32, layers=1)


def parse_ttq(path):
    data = pathlib.Path(path).read_bytes()
    magic, version, model, count, _, dir_off, data_off, layers, experts, dim, vocab = struct.unpack_from(
        "<8sIIIIQQIIII", data, 0)
    recs = []
    for i in range(count):
        off = dir_off + i * 184
        name = data[off:off + 128].split(b"\0")[0].decode()
        fmt, rank = struct.unpack_from("<II", data, off + 128)
        shape = struct.unpack_from("<4Q", data, off + 136)[:rank]
        poff, size = struct.unpack_from("<QQ", data, off + 168)
        recs.append((name, fmt, shape, poff, size, data[poff:poff + size]))
    return (magic, version, model, count, dir_off, data_off, layers, experts, dim, vocab), recs


def test_ttq_writer_roundtrip(tmp_path):
    import ttl_moe
    path = tmp_path / "model.ttq"
    payload_a = np.arange(100, dtype=np.uint8)
    payload_b = np.arange(37, dtype=np.float32)
    with ttl_moe.TtqWriter(path, 20, 24, 32, 2) as w:
        w.add("blk.0.ffn_gate_exps.weight.gpu", ttl_moe.TTQ_FORMAT_MXFP4_GPU, (2880, 2880, 32), payload_a)
        w.add("blk.0.ffn_gate_exps.bias", 1, (2880, 32), payload_b)
        w.finish()
    hdr, recs = parse_ttq(path)
    assert hdr[0] == b"TTLBQNT1" and hdr[1] == 1 and hdr[2] == 20 and hdr[3] == 2
    assert hdr[4] == 56 and hdr[5] % 64 == 0 and hdr[5] >= 56 + 2 * 184
    assert hdr[6:] == (24, 32, 2880, 201088)
    assert recs[0][1] == 6 and recs[0][2] == (2880, 2880, 32)
    for r in recs:
        assert r[3] % 64 == 0
    assert recs[0][5] == payload_a.tobytes()
    assert recs[1][5] == payload_b.tobytes()
    assert not list(tmp_path.glob("*.tmp.*"))


def test_ttq_writer_failure_leaves_target_and_no_temp(tmp_path):
    import ttl_moe
    path = tmp_path / "model.ttq"
    path.write_bytes(b"old contents")
    w = ttl_moe.TtqWriter(path, 20, 24, 32, 2)
    w.add("a", 6, (1,), np.zeros(4, np.uint8))
    with pytest.raises(RuntimeError, match="record count mismatch"):
        w.finish()
    w.close()
    assert path.read_bytes() == b"old contents"  # atomic: target untouched
    assert not list(tmp_path.glob("*.tmp.*"))
    with pytest.raises(RuntimeError, match="only gpt-oss-20b and gpt-oss-120b"):
        ttl_moe.TtqWriter(path, 20, 36, 32, 1)


def test_ttq_writer_reports_write_failure(tmp_path):
    """Fault injection as in tt-lab tests/requant.py:81-103: a file-size limit
    makes the payload write fail; the error surfaces and no temp file stays."""
    script = f"""
import resource, signal, sys
sys.path.insert(0, {str(ROOT / 'tt-lab_b200' / 'python')!r})
signal.signal(signal.SIGXFSZ, signal.SIG_IGN)
resource.setrlimit(resource.RLIMIT_FSIZE, (4096, 4096))
import numpy as np, ttl_moe
w = ttl_moe.TtqWriter({str(tmp_path / 'big.ttq')!r}, 20, 24, 32, 1)
try:
    w.add("x", 6, (1,), np.zeros(1 << 20, np.uint8))
    w.finish()
except RuntimeError as e:
    print("FAILED:", e)
w.close()
"""
    out = subprocess.run(["python", "-c", script], capture_output=True, text=True, timeout=120)
    assert "FAILED" in out.stdout, out.stdout + out.stderr
    assert not (tmp_path / "big.ttq").exists()
    assert not list(tmp_path.glob("*.tmp.*"))


def test_cpp_wrapper_header_compiles(tmp_path):
    src = tmp_path / "t.cpp"
    src.write_text('#include "cuda_moe.hpp"\nint main() { ttl_moe_config c{}; (void)c; return 0; }\n')
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    f"-I{ROOT / 'tt-lab_b200' / 'host'}", str(src)], check=True)
