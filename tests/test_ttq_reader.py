"""The TTQ files this library writes, read back by tt-lab's own reader
(TtqFile, src/tt_backend.cpp:315-445, compiled here from the reference
sources into oracle/_ref/libttlttq.so), and the requant entry's refusals of
GGUF files it cannot convert (checked before any file or GPU is touched)."""
import numpy as np
import pytest

import oracle
from gguf_write import F32, MXFP4, gpt_oss_meta, write_gguf

needs_reader = pytest.mark.skipif(not oracle.ttq_available(), reason="tt-lab TTQ reader not built")


@needs_reader
def test_tt_lab_ttqfile_reads_writer_output(tmp_path):
    import ttl_moe
    path = tmp_path / "m.ttq"
    rng = np.random.default_rng(3)
    recs = [("blk.0.ffn_gate_inp.weight", ttl_moe.TTQ_FORMAT_F32, (2880, 32),
             rng.standard_normal(2880 * 32).astype(np.float32)),
            ("blk.0.ffn_gate_exps.weight.mxfp4gpu", ttl_moe.TTQ_FORMAT_MXFP4_GPU, (2880, 2880, 32),
             rng.integers(0, 256, 1000, dtype=np.uint8)),
            ("blk.0.ffn_gate_exps.bias", ttl_moe.TTQ_FORMAT_F32, (2880, 32),
             rng.standard_normal(77).astype(np.float32))]
    with ttl_moe.TtqWriter(path, 120, 36, 128, len(recs)) as w:
        for r in recs:
            w.add(*r)
        w.finish()
    got = oracle.ttq_read(path)
    assert got.layers == 36 and len(got) == len(recs)
    for g, (name, fmt, shape, payload) in zip(got, recs):
        assert g["name"] == name and g["format"] == fmt and g["shape"] == list(shape)
        assert g["payload"].ctypes.data % 64 == 0  # the mapping is page-aligned, so the offset is too
        assert g["payload"].tobytes() == payload.tobytes()


@needs_reader
def test_tt_lab_ttqfile_rejects_a_truncated_file(tmp_path):
    import ttl_moe
    path = tmp_path / "m.ttq"
    with ttl_moe.TtqWriter(path, 20, 24, 32, 1) as w:
        w.add("x", ttl_moe.TTQ_FORMAT_F32, (4,), np.zeros(4, np.float32))
        w.finish()
    data = path.read_bytes()
    (tmp_path / "cut.ttq").write_bytes(data[:-8])
    with pytest.raises(RuntimeError, match="outside file"):
        oracle.ttq_read(tmp_path / "cut.ttq")


def _requant_error(tmp_path, meta, tensors, layers=(0, 1)):
    import ttl_moe
    src, dst = tmp_path / "m.gguf", tmp_path / "m.ttq"
    write_gguf(src, meta, tensors)
    with pytest.raises(RuntimeError) as e:
        ttl_moe.requant_gpu(src, dst, *layers)
    assert not dst.exists() and not list(tmp_path.glob("*.tmp.*"))
    return str(e.value)


def test_requant_refuses_unconvertible_gguf(tmp_path):
    small = [("blk.0.ffn_gate_inp.weight", F32, [2880, 16], np.zeros(2880 * 16, np.float32))]
    assert "not gpt-oss" in _requant_error(tmp_path, gpt_oss_meta(architecture="llama"), [])
    assert "only gpt-oss-20b and gpt-oss-120b" in _requant_error(tmp_path, gpt_oss_meta(model_layers=12), [])
    assert "bad layer range" in _requant_error(tmp_path, gpt_oss_meta(), [], layers=(3, 25))
    assert "GGUF tensor missing: blk.0.ffn_gate_inp.weight" in _requant_error(tmp_path, gpt_oss_meta(), [])
    assert "unexpected type or shape for GGUF tensor blk.0.ffn_gate_inp.weight" in _requant_error(
        tmp_path, gpt_oss_meta(), small)
    wrong_type = [("blk.0.ffn_gate_inp.weight", MXFP4, [2880, 32], np.zeros(2880 * 17, np.uint8))]
    assert "unexpected type or shape" in _requant_error(tmp_path, gpt_oss_meta(), wrong_type)


def test_requant_refuses_truncated_and_foreign_files(tmp_path):
    import ttl_moe
    src = tmp_path / "m.gguf"
    write_gguf(src, gpt_oss_meta(), [])
    src.write_bytes(src.read_bytes()[:40])
    with pytest.raises(RuntimeError, match="truncated"):
        ttl_moe.requant_gpu(src, tmp_path / "m.ttq", 0, 1)
    (tmp_path / "x.gguf").write_bytes(b"GGML" + bytes(60))
    with pytest.raises(RuntimeError, match="not a GGUF file"):
        ttl_moe.requant_gpu(tmp_path / "x.gguf", tmp_path / "m.ttq", 0, 1)
    with pytest.raises(RuntimeError, match="cannot open GGUF"):
        ttl_moe.requant_gpu(tmp_path / "absent.gguf", tmp_path / "m.ttq", 0, 1)
