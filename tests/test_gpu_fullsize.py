"""Parity at the benchmarked sizes (-m gpu), against tt-lab's compiled CPU code.

  cfg1  gpt-oss-20b, 24 layers x 256 sequential tokens through ttl_moe_forward
        (the bench's headline launch), every one of the 6,144 (token, layer)
        steps checked on the GPU's own input for it (oracle/parity.py), plus
        the free-running 24-layer trajectory of a token sample;
  cfg3  gpt-oss-120b, 36 layers x 4 tokens (128 experts), every step;
  cfg4  gpt-oss-120b layer, prefill T = 2048 with Zipf(1.2)-skewed routing,
        through ttl_moe_prefill against GptOssModel::moe_batch on the whole
        batch (its matvec/matmul choice depends on the batch).

Acceptance: top-4 bit-exact except at near-ties
(reference logits within 1e-6), outputs within max-relative 1e-3.  Weights are
generated on the device by the library's seeded generator and copied to the
host for the checker, one layer at a time.
"""
import numpy as np
import pytest

import oracle
from oracle import parity

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")]


def host(t):
    return {k: v.cpu().numpy() for k, v in t.items()}


def run_stack(E, layers, tokens, seed):
    import torch
    import ttl_moe
    from ttl_moe import synth
    torch.cuda.set_device(0)
    m = ttl_moe.MoE(experts=E, layers=layers, max_tokens=0, device=0)
    for l in range(layers):
        t = synth.layer_device(seed, l, E, device="cuda")
        m.upload_layer(l, t)
        del t
    torch.cuda.empty_cache()
    x = synth.inputs_host(seed, tokens)
    steps = tokens * layers
    ylog = torch.empty((steps, 2880), dtype=torch.float32, device="cuda")
    ilog = torch.empty((steps, 4), dtype=torch.int32, device="cuda")
    wlog = torch.empty((steps, 4), dtype=torch.float32, device="cuda")
    m.record(steps, ylog, ilog, wlog)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    m.forward_async(0, layers, xd, yd, tokens)
    m.sync()
    out = (x, yd.cpu().numpy(), ylog.cpu().numpy().reshape(tokens, layers, 2880),
           ilog.cpu().numpy().reshape(tokens, layers, 4), wlog.cpu().numpy().reshape(tokens, layers, 4))
    m.record(0)
    m.close()
    return out


def layers_from_device(seed, E, layers, keep=None):
    """(layer, host tensors) of the seeded layers, made on the device and
    copied over one at a time; keep: a list the tensors are appended to."""
    from ttl_moe import synth
    for l in range(layers):
        t = host(synth.layer_device(seed, l, E, device="cuda"))
        if keep is not None:
            keep.append(t)
        yield l, t


def free_running(layers_host, x):
    """tt-lab's own token-major forward of the sample tokens (all layers)."""
    return oracle.forward_tokens(layers_host, x)


def test_cfg1_full_stack_parity():
    E, L, T, seed = 32, 24, 256, 0
    x, y, ylog, ilog, wlog = run_stack(E, L, T, seed)
    assert np.array_equal(ylog[:, -1, :], y)
    kept = []
    s = parity.teacher_forced(layers_from_device(seed, E, L, keep=kept), x, ylog, ilog, wlog)
    print("cfg1 teacher-forced:", s)
    assert s["steps"] == T * L
    assert parity.passed(s), s
    assert s["max_w_rel"] <= 1e-5, s
    # free-running 24-layer trajectory of a sample of tokens (none of whose
    # steps hit a near-tie, or the trajectories may part)
    sample = np.arange(0, T, 16)
    yr = free_running(kept, x[sample])
    m = oracle.compare(y[sample], yr)
    print("cfg1 free-running sample:", m)
    assert m["max_rel"] <= 1e-3, m


def test_cfg3_120b_36_layer_parity():
    E, L, T, seed = 128, 36, 4, 3
    x, y, ylog, ilog, wlog = run_stack(E, L, T, seed)
    s = parity.teacher_forced(layers_from_device(seed, E, L), x, ylog, ilog, wlog)
    print("cfg3 teacher-forced:", s)
    assert s["steps"] == T * L
    assert parity.passed(s), s


def test_cfg4_prefill_2048_zipf_parity():
    import torch
    import ttl_moe
    from ttl_moe import synth
    E, T = 128, 2048
    torch.cuda.set_device(0)
    t = synth.layer_device(4, 0, E, device="cuda", zipf_s=1.2)
    th = host(t)
    x = synth.inputs_host(4, T)
    with ttl_moe.MoE(experts=E, layers=1, max_tokens=T, device=0) as m:
        m.upload_layer(0, t)
        del t
        out, idx, w = m.moe_batch(0, x)
    ref, ridx, rw = oracle.moe_prefill(th, x, impl="ref")
    # near-ties are judged on tt-lab's own router logits of the token
    bad = np.nonzero(np.any(idx != ridx, axis=1))[0]
    kinds = {}
    if bad.size:
        lg = oracle.router_logits(th, x[bad])
        kinds = {int(k): parity.classify_top4(idx[k], ridx[k], lg[j]) for j, k in enumerate(bad)}
    assert all(v == "near_tie" for v in kinds.values()), kinds
    good = np.setdiff1d(np.arange(T), bad)
    mm = oracle.compare(out[good], ref[good])
    print("cfg4 prefill: near-ties", len(kinds), mm, "experts hit", np.bincount(ridx.ravel(), minlength=E).max())
    assert mm["max_rel"] <= 1e-3, mm
    assert np.allclose(w[good], rw[good], rtol=1e-5, atol=0)
