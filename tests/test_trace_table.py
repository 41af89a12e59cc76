"""ttl_moe.trace's phase table on a synthetic stamp array (CPU)."""
import numpy as np


def test_phase_table_is_relative_to_each_step_start():
    from ttl_moe.trace import POINTS, phase_table
    steps = 20
    start = np.arange(steps, dtype=np.int64) * 22_000 + 1_000_000
    tr = np.zeros((steps, 10), np.int64)
    offsets = {0: 0, 4: 1900, 1: 2500, 2: 3000, 3: 9000, 8: 11000, 5: 13000, 6: 17000, 9: 19000, 7: 21900}
    for i, off in offsets.items():
        tr[:, i] = start + off
    t = phase_table(tr, skip=2)
    assert abs(t["step_us"]["mean"] - 22.0) < 1e-9
    for i, name in POINTS.items():
        assert abs(t[name]["median"] - offsets[i] / 1e3) < 1e-9
