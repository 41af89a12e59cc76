"""Token-sharded expert-parallel prefill on CPU: two gloo ranks (127.0.0.1).

Restates, with the oracle's C restatement of tt-lab for the expert math, the
dispatch the library runs between GPUs (tt-lab_b200/csrc/prefill_ep.cu):
each rank routes its own share of the tokens, sends each token once to every
rank owning one of its experts (in token order, with its top-4), the owner
computes its experts over the tokens it received, returns one row w * down
(rounded) per pair in the sender's order and in rank order of the token's
top-4, and the token's owner adds its four rows in ascending expert id.

Each expert's owner receives exactly the tokens tt-lab's moe_batch routes to
that expert, in the same order (the shards are contiguous and arrive in rank
order), so it takes the same matvec / matmul path
(src/model.cpp:396-448) and the combined rows equal tt-lab's moe_batch output
bit for bit (src/model.cpp:450-459).
"""
import ctypes
import json
import pathlib
import socket

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[1]
EXPERTS = 8
TOKENS = 24
D = 2880
MATRIX = D * 90 * 17
SELECTED_MAX = 4  # src/model.cpp:22: up to 4 tokens take the matvec path


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expert_rows(t, e, xs):
    """tt-lab's expert e (gate, up, SwiGLU, down) over the token rows xs, in
    order, by the matvec or the selected-matmul path as moe_batch picks."""
    import oracle
    P = oracle.port()
    n = xs.shape[0]
    gate = np.empty((n, D), np.float32)
    up = np.empty((n, D), np.float32)
    down = np.empty((n, D), np.float32)
    wb = [(t[k + "_w"].ctypes.data + e * MATRIX, t[k + "_b"].ctypes.data + e * D * 4) for k in ("gate", "up", "down")]

    def product(which, inp, out):
        w, b = wb[which]
        if n <= SELECTED_MAX:
            for s in range(n):
                P.oref_matvec_add_mxfp4(w, b, inp[s].ctypes.data, out[s].ctypes.data, oracle.ISA_V4)
        else:
            xt = np.ascontiguousarray(inp.T)
            rows = np.arange(n, dtype=np.uintp)
            P.oref_matmul_add_mxfp4_selected(w, b, xt.ctypes.data, rows.ctypes.data, n, out.ctypes.data,
                                             oracle.ISA_V4)

    product(0, xs, gate)
    product(1, xs, up)
    hidden = np.array([[P.oref_swiglu(ctypes.c_float(a), ctypes.c_float(b)) for a, b in zip(g, u)]
                       for g, u in zip(gate, up)], np.float32)
    product(2, hidden, down)
    return down


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tt-lab_b200" / "python"))
    import datetime
    import torch
    import torch.distributed as dist
    import oracle
    from ttl_moe import synth
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    per = EXPERTS // world
    t = synth.layer_host(7, 0, EXPERTS)
    x_all = synth.inputs_host(8, TOKENS)
    lo, hi = rank * TOKENS // world, (rank + 1) * TOKENS // world
    x = np.ascontiguousarray(x_all[lo:hi])
    _, idx, w = oracle.moe_prefill(t, x, impl="port")  # the router part: per token
    # plan: per destination, the own tokens with an expert there, in token order
    send = [[k for k in range(x.shape[0]) if any(int(e) // per == d for e in idx[k])] for d in range(world)]
    counts = torch.tensor([len(s) for s in send], dtype=torch.int64)
    table = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(table, counts)
    recv_n = [int(table[s][rank]) for s in range(world)]

    def exchange(blocks, shape_of, dtype):
        """blocks[d]: what this rank sends to d; returns what each rank sent here."""
        got = [None] * world
        reqs = []
        for d in range(world):
            if d == rank:
                got[d] = blocks[d]
                continue
            reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(blocks[d])), d))
            buf = torch.empty(shape_of(d), dtype=dtype)
            reqs.append(dist.irecv(buf, d))
            got[d] = buf
        for r in reqs:
            r.wait()
        return [g.numpy() if isinstance(g, torch.Tensor) else g for g in got]

    rows_in = exchange([x[s] for s in send], lambda s: (recv_n[s], D), torch.float32)
    idx_in = exchange([idx[s].astype(np.int64) for s in send], lambda s: (recv_n[s], 4), torch.int64)
    w_in = exchange([w[s] for s in send], lambda s: (recv_n[s], 4), torch.float32)
    rx = np.concatenate(rows_in)
    ridx = np.concatenate(idx_in)
    rw = np.concatenate(w_in)
    # this rank's experts over the received tokens (receive order = token order)
    wdown = {}
    for e in range(rank * per, (rank + 1) * per):
        sel = [j for j in range(rx.shape[0]) if e in ridx[j]]
        if not sel:
            continue
        down = _expert_rows(t, e, rx[sel])
        for s, j in enumerate(sel):
            q = list(ridx[j]).index(e)
            wdown[(j, q)] = (np.float32(rw[j, q]) * down[s]).astype(np.float32)
    # return: per source, its tokens in its send order, local pairs in rank order
    starts = np.cumsum([0] + recv_n)
    back_blocks = []
    for s in range(world):
        rows = [wdown[(j, q)] for j in range(starts[s], starts[s + 1]) for q in range(4)
                if int(ridx[j][q]) // per == rank]
        back_blocks.append(np.array(rows, np.float32).reshape(-1, D))
    pair_n = [sum(1 for k in send[d] for e in idx[k] if int(e) // per == d) for d in range(world)]
    back = exchange(back_blocks, lambda d: (pair_n[d], D), torch.float32)
    # owner combine: ascending expert id, the rows as they came back
    out = np.zeros_like(x)
    for k in range(x.shape[0]):
        rowof = {}
        for d in range(world):
            if k in send[d]:
                before = sum(1 for kk in send[d][:send[d].index(k)] for e in idx[kk] if int(e) // per == d)
                mine = [q for q in range(4) if int(idx[k][q]) // per == d]
                for i, q in enumerate(mine):
                    rowof[int(idx[k][q])] = back[d][before + i]
        acc = np.zeros(D, np.float32)
        for e in sorted(rowof):
            acc = (acc + rowof[e]).astype(np.float32)
        out[k] = acc
    ref, ref_idx, _ = oracle.moe_prefill(t, x_all, impl="port")
    res = {"rank": rank, "exact": bool(np.array_equal(out, ref[lo:hi])),
           "idx_ok": bool(np.array_equal(idx, ref_idx[lo:hi])),
           "max_abs": float(np.max(np.abs(out - ref[lo:hi]))), "sent": [len(s) for s in send]}
    (pathlib.Path(outdir) / f"rank{rank}.json").write_text(json.dumps(res))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_token_sharded_prefill(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0, f"rank process exited with {p.exitcode}"
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    for r in res:
        assert r["idx_ok"], r
        assert r["exact"], r
        assert sum(r["sent"]) > 0
