"""tt-lab's own GptOssModel::prefill and forward with the MoE on the GPU
(oracle/_ref/ttlab_cuda_check, built from oracle/cuda_check.cpp): the
compiled binding, its hook bound to tt-lab's calls at src/model.cpp:536 and
:591 without editing tt-lab, checked against the same model on the CPU with
run_device_proxy_check's metrics (src/tt_backend.cpp:3647-3714)."""
import json
import pathlib
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
BIN = ROOT / "oracle" / "_ref" / "ttlab_cuda_check"

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not BIN.exists(), reason="oracle/_ref/ttlab_cuda_check not built")]


def test_tt_lab_forward_with_the_cuda_moe():
    prompt, generate = 8, 4
    r = subprocess.run([str(BIN), str(prompt), str(generate), "0"], capture_output=True, text=True, timeout=900)
    print(r.stdout)
    assert r.returncode == 0, r.stderr
    m = json.loads(r.stdout.strip().splitlines()[-1])
    layers = 24
    # every MoE call of tt-lab's prefill (one moe_batch per layer) and of its
    # generation (one moe per layer per token) went to the GPU
    assert m["gpu_moe_calls"] == layers * (1 + generate)
    assert m["selections"] == layers * (prompt + generate)
    # the two models' residual streams part by f32 rounding (the MoE sums in
    # another order), so an occasional near-tie routes differently: the bar
    # is the proxy check's kind -- near-total agreement, not bit equality
    assert m["top4_overlap_avg"] >= 3.95 and m["top1_match"] >= 0.97, m
    assert m["moe_close"] >= 0.95 * m["selections"], m
    assert m["logits_cosine_min"] > 0.999 and m["greedy_matches"] == m["greedy_total"], m
