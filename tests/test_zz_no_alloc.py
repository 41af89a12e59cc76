"""ttl_matvec_mxfp4_noalloc: the allocation-free variant of ttl_matvec_mxfp4
(scratch in a fixed static device array).  Kept in its own file, collected
last, so it runs both alone and after every other test of the session."""
import numpy as np
import pytest

D = 2880


def test_noalloc_refuses_more_than_its_scratch_before_touching_the_gpu():
    import ttl_moe
    buf = np.zeros(16, np.float32)  # never dereferenced: the count is checked first
    with pytest.raises(RuntimeError, match="1..256 matrices per call"):
        ttl_moe.matvec_mxfp4_noalloc(buf, buf, buf, buf, matrices=257)
    with pytest.raises(RuntimeError, match="1..256 matrices per call"):
        ttl_moe.matvec_mxfp4_noalloc(buf, buf, buf, buf, matrices=0)


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_on_consecutive_calls():
    import torch
    import ttl_moe
    from conftest import synth_layer
    from ttl_moe import synth
    t = synth_layer(0, 32)
    M = 3
    g = torch.from_numpy(np.ascontiguousarray(t["down_w"][: M * D * 90 * 17])).cuda()
    packed = torch.empty(ttl_moe.packed_bytes(M), dtype=torch.uint8, device="cuda")
    ttl_moe.pack_mxfp4(g, M, packed)
    bias = torch.from_numpy(np.ascontiguousarray(t["down_b"][: M * D])).cuda()
    for call in range(2):  # two consecutive calls: the scratch starts at zero each time
        x = torch.from_numpy(synth.inputs_host(40 + call, M).ravel().copy()).cuda()
        y_ref = torch.empty(M * D, device="cuda")
        for m in range(M):
            ttl_moe.matvec_mxfp4(packed[m * ttl_moe.packed_bytes(1):], bias[m * D:], x[m * D:], y_ref[m * D:])
        y = torch.full((M * D,), float("nan"), device="cuda")
        ttl_moe.matvec_mxfp4_noalloc(packed, bias, x, y, matrices=M)
        assert torch.equal(y, y_ref)
        y1 = torch.full((D,), float("nan"), device="cuda")
        ttl_moe.matvec_mxfp4_noalloc(packed, bias, x, y1, matrices=1)
        assert torch.equal(y1, y_ref[:D])


@pytest.mark.gpu
def test_noalloc_full_scratch_and_stale_status_words():
    """256 matrices (the whole scratch; three packed matrices repeated into
    one buffer) against the allocating entry, then a smaller call right after
    it on the same scratch (the entry zeroes the status words it uses on every
    call)."""
    import torch
    import ttl_moe
    from conftest import synth_layer
    from ttl_moe import synth
    t = synth_layer(0, 32)
    P = ttl_moe.packed_bytes(1)
    g = torch.from_numpy(np.ascontiguousarray(t["up_w"][: 3 * D * 90 * 17])).cuda()
    three = torch.empty(ttl_moe.packed_bytes(3), dtype=torch.uint8, device="cuda")
    ttl_moe.pack_mxfp4(g, 3, three)
    M = 256
    packed = three.view(3, P).repeat(M // 3 + 1, 1)[:M].contiguous().view(-1)
    bias = torch.from_numpy(np.ascontiguousarray(t["up_b"][: 3 * D])).cuda().view(3, D).repeat(M // 3 + 1, 1)[:M]
    bias = bias.contiguous().view(-1)
    x = torch.from_numpy(synth.inputs_host(50, M).ravel().copy()).cuda()
    y = torch.full((M * D,), float("nan"), device="cuda")
    ttl_moe.matvec_mxfp4_noalloc(packed, bias, x, y, matrices=M)
    for m in (0, 1, 2, 127, 254, 255):
        y_ref = torch.empty(D, device="cuda")
        ttl_moe.matvec_mxfp4(packed[m * P:], bias[m * D:], x[m * D:], y_ref)
        assert torch.equal(y[m * D:(m + 1) * D], y_ref), m
    y2 = torch.full((2 * D,), float("nan"), device="cuda")
    ttl_moe.matvec_mxfp4_noalloc(packed, bias, x, y2, matrices=2)
    assert torch.equal(y2, y[: 2 * D])
