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
