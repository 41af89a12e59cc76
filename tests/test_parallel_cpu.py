"""Expert parallelism on CPU: two gloo ranks (world size 2, 127.0.0.1).

Checks the host-side plumbing the multi-GPU launch uses (ttl_moe.parallel:
expert partition, NCCL-id broadcast, max-over-ranks timing) and the
decomposition the library's expert-parallel decode relies on: each rank runs
the replicated router, computes the weighted down outputs of the selected
experts it owns, and the sum over ranks equals tt-lab's rank-order combine
(src/model.cpp:323-336) up to f32 reassociation.  The expert math is the
oracle's C restatement of tt-lab (no GPU involved).
"""
import json
import pathlib
import socket

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
EXPERTS = 8
D = 2880
MATRIX = D * 90 * 17


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial_decode(t, x, lo, hi):
    """Weighted down outputs of the selected experts in [lo, hi), in rank order."""
    import ctypes
    import oracle
    P = oracle.port()
    full, idx, w = oracle.moe_decode(t, x, impl="port")
    out = np.zeros(D, np.float32)
    g = np.empty(D, np.float32)
    u = np.empty(D, np.float32)
    dn = np.empty(D, np.float32)
    for q in range(4):
        e = int(idx[q])
        if not lo <= e < hi:
            continue
        P.oref_matvec_add_mxfp4(t["gate_w"].ctypes.data + e * MATRIX, t["gate_b"].ctypes.data + e * D * 4,
                                x.ctypes.data, g.ctypes.data, oracle.ISA_V4)
        P.oref_matvec_add_mxfp4(t["up_w"].ctypes.data + e * MATRIX, t["up_b"].ctypes.data + e * D * 4,
                                x.ctypes.data, u.ctypes.data, oracle.ISA_V4)
        h = np.array([P.oref_swiglu(ctypes.c_float(a), ctypes.c_float(b)) for a, b in zip(g, u)], np.float32)
        P.oref_matvec_add_mxfp4(t["down_w"].ctypes.data + e * MATRIX, t["down_b"].ctypes.data + e * D * 4,
                                h.ctypes.data, dn.ctypes.data, oracle.ISA_V4)
        out = (out + w[q] * dn).astype(np.float32)
    return out, full, idx


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))
    import datetime
    import torch
    import torch.distributed as dist
    from ttl_moe import parallel, synth
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    res = {"rank": rank}
    lo, hi = parallel.expert_range(rank, world, EXPERTS)
    res["range"] = [lo, hi]
    payload = bytes(range(128)) if rank == 0 else None
    res["shared_ok"] = parallel.share_bytes(dist, payload, 128) == bytes(range(128))
    res["max"] = parallel.max_over_ranks(dist, [float(rank), -float(rank)])
    t = synth.layer_host(5, 0, EXPERTS)
    xs = synth.inputs_host(6, 3)
    errs, zero_when_unowned = [], True
    for k in range(xs.shape[0]):
        x = np.ascontiguousarray(xs[k])
        part, full, idx = _partial_decode(t, x, lo, hi)
        if not any(lo <= int(e) < hi for e in idx):
            zero_when_unowned = zero_when_unowned and not part.any()
        tot = torch.from_numpy(part.copy())
        dist.all_reduce(tot)
        # the library adds the ranks' partials; the reference sums in rank order
        errs.append(float(np.max(np.abs(tot.numpy().astype(np.float64) - full)) / np.max(np.abs(full))))
    res["errs"] = errs
    res["zero_when_unowned"] = zero_when_unowned
    (pathlib.Path(outdir) / f"rank{rank}.json").write_text(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


def test_expert_range_partitions():
    from ttl_moe import parallel
    for world in (1, 2, 4, 8):
        covered = []
        for r in range(world):
            lo, hi = parallel.expert_range(r, world, 32)
            covered += list(range(lo, hi))
        assert covered == list(range(32))
    with pytest.raises(ValueError):
        parallel.expert_range(0, 3, 32)


def test_two_gloo_ranks_expert_parallel_decode(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank process exited with {p.exitcode}"
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    assert [r["range"] for r in res] == [[0, 4], [4, 8]]
    assert all(r["shared_ok"] for r in res)
    assert all(r["max"] == [1.0, 0.0] for r in res)
    for r in res:
        assert r["zero_when_unowned"]
        assert max(r["errs"]) <= 1e-6, r["errs"]
