"""The step-by-step parity checker (oracle/parity.py) on CPU: a log made by
tt-lab's own code passes with zero error, and mistakes planted in that log
(on the CPU) are caught -- a wrong output row, a wrong top-4 that is not a
near-tie -- while a swap of two experts whose logits tie is accepted."""
import numpy as np
import pytest

import oracle
from oracle import parity
from oracle import synth as osynth

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def stack():
    layers = [osynth.layer_host(0, l, 32) for l in range(2)]
    x = osynth.inputs_host(0, 3)
    T, L = 3, 2
    ylog = np.empty((T, L, 2880), np.float32)
    ilog = np.empty((T, L, 4), np.int32)
    wlog = np.empty((T, L, 4), np.float32)
    h = x
    for l in range(L):
        h, idx, w, _ = oracle.moe_layer_tokens(layers[l], h, threads=2)
        ylog[:, l], ilog[:, l], wlog[:, l] = h, idx, w
    return layers, x, ylog, ilog, wlog


def check(stack, ylog=None, ilog=None):
    layers, x, y0, i0, w0 = stack
    return parity.teacher_forced(enumerate(layers), x, y0 if ylog is None else ylog, i0 if ilog is None else ilog,
                                 w0)


def test_reference_log_passes(stack):
    s = check(stack)
    assert parity.passed(s) and s["max_rel"] == 0.0 and s["match"] == 6, s


def test_planted_output_error_is_caught(stack):
    y = stack[2].copy()
    y[1, 1, 100] *= 1.01
    s = check(stack, ylog=y)
    assert not parity.passed(s) and s["worst_step"] == [1, 1], s


def test_planted_selection_error_is_caught(stack):
    idx = stack[3].copy()
    idx[2, 0, 1] = (idx[2, 0, 1] + 1) % 32
    if idx[2, 0, 1] in idx[2, 0, [0, 2, 3]]:
        idx[2, 0, 1] = (idx[2, 0, 1] + 1) % 32
    s = check(stack, ilog=idx)
    assert s["mismatches"] == 1 and not parity.passed(s), s


def test_near_tie_rule():
    logits = np.zeros(32, np.float32)
    logits[[1, 2, 3, 4, 5]] = [3.0, 2.0, 1.0, 0.5, 0.5 + 4e-7]
    assert parity.classify_top4([1, 2, 3, 5], [1, 2, 3, 4], logits) == "near_tie"
    assert parity.classify_top4([1, 3, 2, 4], [1, 2, 3, 4], logits) == "mismatch"
    assert parity.classify_top4([1, 2, 3, 4], [1, 2, 3, 4], logits) == "match"
