"""Expert parallelism on two GPUs (TTL_TEST_WORLD=4 or 8: that many), one
process per GPU (skipped with fewer).

Each rank owns 1/world of the experts.  Decode and forward run in the
persistent kernel: every rank computes the selected experts it owns, and the
ranks exchange their partial output rows inside the kernel over NVLink (peer
stores of tagged words into each other's buffers), adding them in rank order.
So all ranks return the same bits, and those match tt-lab's CPU MoE (the
oracle) within the same tolerance as one GPU.  Prefill is token-sharded:
each rank passes its own share of the tokens, which go to their experts'
owners and come back as weighted rows, all by peer stores into the ranks'
IPC-mapped receive blocks.  The processes
exchange the NCCL id over gloo (127.0.0.1).
"""
import json
import os
import pathlib
import socket

import numpy as np
import pytest

import oracle
from conftest import synth_layer

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]
TOL = 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))
    import datetime
    import torch
    import torch.distributed as dist
    import ttl_moe
    from ttl_moe import parallel, synth
    from conftest import synth_layer as layer_of
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    nid = parallel.share_bytes(dist, ttl_moe.nccl_id() if rank == 0 else None, ttl_moe.NCCL_ID_BYTES)
    layers = [layer_of(40 + l, 32, layer=l, norm=True) for l in range(2)]
    xs = synth.inputs_host(41, 3)
    xp = synth.inputs_host(42, 17)
    lo, hi = (rank * xp.shape[0]) // world, ((rank + 1) * xp.shape[0]) // world
    res = {"rank": rank}
    with ttl_moe.MoE(experts=32, layers=2, max_tokens=32, device=rank, rank=rank, world=world,
                     nccl_id_bytes=nid) as m:
        for l, t in enumerate(layers):
            m.upload_layer(l, t)
        res["persistent"] = m.counters()["persistent_decode"]
        y = m.forward(0, 2, xs)
        y2 = m.forward(0, 2, xs[::-1].copy())  # a replay of the captured forward with new inputs
        out, idx, w = m.moe(0, np.ascontiguousarray(xs[0]))
        pout, pidx, pw = m.moe_batch(0, xp[lo:hi])
    np.save(pathlib.Path(outdir) / f"y{rank}.npy", y)
    np.save(pathlib.Path(outdir) / f"y2_{rank}.npy", y2)
    np.save(pathlib.Path(outdir) / f"d{rank}.npy", out)
    np.save(pathlib.Path(outdir) / f"p{rank}.npy", pout)
    res["idx"] = [int(v) for v in idx]
    res["pidx"] = pidx.tolist()
    (pathlib.Path(outdir) / f"rank{rank}.json").write_text(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


def _rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b)))


def test_two_gpu_expert_parallel_matches_reference(tmp_path):
    import torch
    world = int(os.environ.get("TTL_TEST_WORLD", "2"))
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0, f"rank process exited with {p.exitcode}"
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    assert all(r["persistent"] == 1 for r in res), res
    from ttl_moe import synth
    layers = [synth_layer(40 + l, 32, layer=l, norm=True) for l in range(2)]
    xs = synth.inputs_host(41, 3)
    xp = synth.inputs_host(42, 17)
    impl = "ref" if oracle.ref_available() else "port"
    ys = [np.load(tmp_path / f"y{r}.npy") for r in range(world)]
    y2s = [np.load(tmp_path / f"y2_{r}.npy") for r in range(world)]
    ds = [np.load(tmp_path / f"d{r}.npy") for r in range(world)]
    ps = [np.load(tmp_path / f"p{r}.npy") for r in range(world)]
    # the ranks add the same partials in the same order
    for r in range(1, world):
        assert np.array_equal(ys[0], ys[r]) and np.array_equal(y2s[0], y2s[r]) and np.array_equal(ds[0], ds[r])
    ry = oracle.forward(layers, xs, impl=impl)
    ry2 = oracle.forward(layers, xs[::-1].copy(), impl=impl)
    for k in range(3):
        assert _rel(ys[0][k], ry[k]) <= TOL
        assert _rel(y2s[0][k], ry2[k]) <= TOL
    rd, ridx, _ = oracle.moe_decode(layers[0], np.ascontiguousarray(xs[0]), impl=impl)
    assert all(r["idx"] == [int(v) for v in ridx] for r in res)
    assert _rel(ds[0], rd) <= TOL
    rp, rpidx, _ = oracle.moe_prefill(layers[0], xp, impl=impl)
    n = xp.shape[0]
    assert sum((res[r]["pidx"] for r in range(world)), []) == rpidx.tolist()
    for r in range(world):
        lo, hi = (r * n) // world, ((r + 1) * n) // world
        assert _rel(ps[r], rp[lo:hi]) <= TOL


def _fault_worker(rank, world, port, outdir):
    """One rank rejects a decode call on the host while its peers launch (their
    kernels' bounded waits for it run out after 2 s); every rank's next call
    is refused until all have called resync, after which decode and forward
    agree again.  Then rank 1 skips a prefill: rank 0's waits for its rows
    run out on the device, and after a resync prefill agrees again.  The
    processes meet on gloo between steps; each step is logged to a file so
    that a stuck rank shows where it stopped."""
    import sys
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))
    import datetime
    import torch
    import torch.distributed as dist
    import ttl_moe
    from ttl_moe import parallel, synth
    from conftest import synth_layer as layer_of
    log = open(pathlib.Path(outdir) / f"log{rank}.txt", "w", buffering=1)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    nid = parallel.share_bytes(dist, ttl_moe.nccl_id() if rank == 0 else None, ttl_moe.NCCL_ID_BYTES)
    layers = [layer_of(40 + l, 32, layer=l, norm=True) for l in range(2)]
    xs = synth.inputs_host(41, 3)
    x = np.ascontiguousarray(xs[0])
    res = {"rank": rank}

    def attempt(key, fn):
        log.write(f"{key}: start\n")
        try:
            fn()
            res[key] = "ok"
        except RuntimeError as e:
            res[key] = str(e)
        log.write(f"{key}: {res[key]}\n")

    with ttl_moe.MoE(experts=32, layers=2, max_tokens=16, device=rank, rank=rank, world=world,
                     nccl_id_bytes=nid) as m:
        for l, t in enumerate(layers):
            m.upload_layer(l, t)
        m.set_timeout(30000)
        before = m.moe(0, x)[0]
        log.write("before: ok\n")
        dist.barrier()
        attempt("rejected", lambda: m.moe(0 if rank == 0 else 99, x))
        attempt("refused", lambda: m.moe(0, x))
        attempt("resync", m.resync)
        after = m.moe(0, x)[0]
        y = m.forward(0, 2, xs)
        log.write("after: ok\n")
        res["decode_same"] = bool(np.array_equal(before, after))
        np.save(pathlib.Path(outdir) / f"f{rank}.npy", after)
        np.save(pathlib.Path(outdir) / f"fy{rank}.npy", y)
        dist.barrier()
        # prefill: rank 1 skips a call; rank 0's waits for its rows and its
        # done flag run out on the device (2 s each), and rank 0 fails
        xp = synth.inputs_host(42, 16)
        lo, hi = (rank * 16) // world, ((rank + 1) * 16) // world
        p_before = m.moe_batch(0, xp[lo:hi])[0]
        log.write("prefill: ok\n")
        if rank == 0:
            attempt("prefill_alone", lambda: m.moe_batch(0, xp[lo:hi]))
        dist.barrier()  # the host control plane tells every rank
        attempt("prefill_resync", m.resync)
        p_after = m.moe_batch(0, xp[lo:hi])[0]
        res["prefill_same"] = bool(np.array_equal(p_before, p_after))
        np.save(pathlib.Path(outdir) / f"fp{rank}.npy", p_after)
        dist.barrier()
    log.write("closed\n")
    (pathlib.Path(outdir) / f"fault{rank}.json").write_text(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


def test_expert_parallel_failure_and_resync(tmp_path, monkeypatch):
    import torch
    world = int(os.environ.get("TTL_TEST_WORLD", "2"))
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")  # no NVLink multicast objects while a rank may fail
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, world, port, str(tmp_path)), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    stuck = [r for r, p in enumerate(procs) if p.exitcode is None]
    for p in procs:
        if p.exitcode is None:
            p.kill()
            p.join(timeout=30)
    logs = {r: (tmp_path / f"log{r}.txt").read_text() if (tmp_path / f"log{r}.txt").exists() else ""
            for r in range(world)}
    assert not stuck, f"ranks {stuck} did not finish; logs: {logs}"
    assert all(p.exitcode == 0 for p in procs), ([p.exitcode for p in procs], logs)
    res = [json.loads((tmp_path / f"fault{r}.json").read_text()) for r in range(world)]
    # the rank that rejected the call, and the peers whose kernels waited for it, all fail
    assert "bounded-wait-timeout" in res[0]["rejected"], res[0]
    for r in range(1, world):
        assert "out of range" in res[r]["rejected"], res[r]
    for r in res:
        assert "ttl_moe_resync" in r["refused"], r
        assert r["resync"] == "ok" and r["decode_same"], r
    fs = [np.load(tmp_path / f"f{r}.npy") for r in range(world)]
    fys = [np.load(tmp_path / f"fy{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(fs[0], fs[r]) and np.array_equal(fys[0], fys[r])
    from ttl_moe import synth
    layers = [synth_layer(40 + l, 32, layer=l, norm=True) for l in range(2)]
    xs = synth.inputs_host(41, 3)
    impl = "ref" if oracle.ref_available() else "port"
    rd, _, _ = oracle.moe_decode(layers[0], np.ascontiguousarray(xs[0]), impl=impl)
    assert _rel(fs[0], rd) <= TOL
    ry = oracle.forward(layers, xs, impl=impl)
    for k in range(3):
        assert _rel(fys[0][k], ry[k]) <= TOL
    # prefill after the failed call and the resync
    assert "bounded-wait-timeout" in res[0]["prefill_alone"], res[0]
    for r in res:
        assert r["prefill_resync"] == "ok" and r["prefill_same"], r
    xp = synth.inputs_host(42, 16)
    rp, _, _ = oracle.moe_prefill(layers[0], xp, impl=impl)
    for r in range(world):
        lo, hi = (r * 16) // world, ((r + 1) * 16) // world
        assert _rel(np.load(tmp_path / f"fp{r}.npy"), rp[lo:hi]) <= TOL
