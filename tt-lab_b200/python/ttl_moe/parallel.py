"""Host-side plumbing of expert parallelism (one process per GPU).

The library partitions experts the same way (ttl_moe_create: rank r owns
experts [r*E/world, (r+1)*E/world)); every rank runs the replicated router
and computes the weighted down outputs of the selected experts it owns, and
the ranks sum them (NCCL all-reduce inside the library).  These helpers are
the torch.distributed side a launcher needs around it: sharing the library's
NCCL id and reducing timings.  They work with any backend (NCCL on GPUs,
gloo on CPU).
"""
from __future__ import annotations


def expert_range(rank: int, world: int, experts: int) -> tuple[int, int]:
    """Experts [lo, hi) owned by `rank` (world must divide experts)."""
    if world <= 0 or experts % world != 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world} cannot split {experts} experts evenly")
    per = experts // world
    return rank * per, (rank + 1) * per


def share_bytes(dist, payload: bytes | None, nbytes: int, device="cpu") -> bytes:
    """Broadcasts rank 0's `payload` (exactly nbytes) to every rank."""
    import torch
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
    if dist.get_rank() == 0:
        if payload is None or len(payload) != nbytes:
            raise ValueError(f"rank 0 must provide {nbytes} bytes")
        buf.copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
    dist.broadcast(buf, 0)
    return bytes(buf.cpu().numpy().tobytes())


def max_over_ranks(dist, values, device="cpu"):
    """Element-wise maximum of a list of floats over all ranks."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]
