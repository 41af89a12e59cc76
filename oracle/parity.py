"""Step-by-step parity of the GPU decode against tt-lab's compiled CPU code --
TEST INFRASTRUCTURE ONLY (the checker; tests/ and bench.py's parity sample,
outside any timed region).

The GPU's persistent kernel logs every (token, layer) step it runs: its output
row and its top-4 (ttl_moe_record).  Each step is replayed here through
tt-lab's own rms_norm + GptOssModel::moe + residual (oracle/_ref) on the GPU's
own input for that step -- the token's input on layer 0, the GPU's output of the
previous layer after that -- so every step is compared on identical inputs
("teacher forcing"), and one near-tie cannot spread into the later layers.

Acceptance: the top-4 indices equal the reference's
except at near-ties, where every expert the two lists place differently has a
reference logit within 1e-6 of the expert the reference placed there; the
output agrees to max |y - y_ref| / max |y_ref| <= 1e-3 on every step whose
top-4 matched.
"""
from __future__ import annotations

import numpy as np

from . import moe_layer_tokens

TIE = 1.0e-6
TOL = 1.0e-3


def classify_top4(gpu_idx, ref_idx, ref_logits, tie=TIE):
    """'match', 'near_tie' or 'mismatch' for one step's ordered top-4."""
    g = np.asarray(gpu_idx).ravel()
    r = np.asarray(ref_idx).ravel()
    if np.array_equal(g, r):
        return "match"
    for a, b in zip(g, r):
        if a != b and not (abs(float(ref_logits[a]) - float(ref_logits[b])) < tie):
            return "mismatch"
    return "near_tie"


def teacher_forced(layer_iter, x, y_log, idx_log, w_log, threads=None, norms=None):
    """x [T, 2880] the tokens' inputs; y_log [T, L, 2880], idx_log / w_log
    [T, L, 4] the GPU's step log; layer_iter yields (layer, host tensors) in
    layer order, one layer at a time.  Returns the summary dict (and raises
    nothing: the caller asserts)."""
    T, L = y_log.shape[0], y_log.shape[1]
    out = {"steps": 0, "max_rel": 0.0, "match": 0, "near_ties": 0, "mismatches": 0, "max_w_rel": 0.0,
           "worst_step": None, "mismatch_steps": []}
    for l, t in layer_iter:
        inp = x if l == 0 else y_log[:, l - 1, :]
        g = None if norms is None else norms[l]
        y_ref, idx_ref, w_ref, logits = moe_layer_tokens(t, np.ascontiguousarray(inp), norm_w=g, threads=threads)
        for k in range(T):
            kind = classify_top4(idx_log[k, l], idx_ref[k], logits[k])
            out["steps"] += 1
            if kind == "match":
                out["match"] += 1
                ref = y_ref[k].astype(np.float64)
                err = np.max(np.abs(y_log[k, l].astype(np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30)
                if err > out["max_rel"]:
                    out["max_rel"] = float(err)
                    out["worst_step"] = [int(k), int(l)]
                wr = np.max(np.abs(w_log[k, l].astype(np.float64) - w_ref[k]) / np.abs(w_ref[k]))
                out["max_w_rel"] = max(out["max_w_rel"], float(wr))
            elif kind == "near_tie":
                out["near_ties"] += 1
            else:
                out["mismatches"] += 1
                if len(out["mismatch_steps"]) < 8:
                    out["mismatch_steps"].append([int(k), int(l), idx_log[k, l].tolist(), idx_ref[k].tolist()])
    return out


def passed(summary, tol=TOL):
    return summary["mismatches"] == 0 and summary["max_rel"] <= tol and summary["steps"] > 0
