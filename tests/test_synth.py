"""The synthetic-input generator (csrc/synth.h) against an independent numpy
twin, and the distributions BASELINE.json asks for."""
import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def mix(z):
    z = np.asarray(z, np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def key(seed, stream):
    with np.errstate(over="ignore"):
        a = mix(np.uint64(seed) + np.uint64(0x9E3779B97F4A7C15))
        b = np.uint64(stream) * np.uint64(0xD1B54A32D192ED03) + np.uint64(1)
    return mix(a ^ b)


def draw(k, i):
    with np.errstate(over="ignore"):
        return mix(k + (np.asarray(i, np.uint64) + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15))


def twin_normal(n, seed, stream, sigma):
    k = key(seed, stream)
    i = np.arange(n, dtype=np.uint64)
    total = np.zeros(n, np.int64)
    for j in range(6):
        h = draw(k, i * np.uint64(6) + np.uint64(j))
        total += (h & np.uint64(0xFFFFFF)).astype(np.int64) + ((h >> np.uint64(32)) & np.uint64(0xFFFFFF)).astype(np.int64)
    v = (total - 100663296).astype(np.int32).astype(np.float32) * np.float32(2.0 ** -24)
    return (v * np.float32(sigma)).astype(np.float32)


def twin_mxfp4(blocks, seed, stream, lo, count):
    k = key(seed, stream)
    b = np.arange(blocks, dtype=np.uint64)
    h0 = draw(k, b * np.uint64(3))
    h1 = draw(k, b * np.uint64(3) + np.uint64(1))
    h2 = draw(k, b * np.uint64(3) + np.uint64(2))
    out = np.empty((blocks, 17), np.uint8)
    with np.errstate(over="ignore"):
        out[:, 0] = (lo + (((h2 >> np.uint64(32)) * np.uint64(count)) >> np.uint64(32))).astype(np.uint8)
    out[:, 1:9] = h0.view(np.uint8).reshape(blocks, 8)
    out[:, 9:17] = h1.view(np.uint8).reshape(blocks, 8)
    return out.reshape(-1)


def test_normal_matches_twin():
    from ttl_moe import synth
    a = synth.normal_host(5000, 3, 17, 0.02)
    b = twin_normal(5000, 3, 17, 0.02)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_mxfp4_matches_twin():
    from ttl_moe import synth
    a = synth.mxfp4_host(3000, 5, 2)
    b = twin_mxfp4(3000, 5, 2, 119, 7)
    assert np.array_equal(a, b)


def test_distributions():
    from ttl_moe import synth
    x = synth.normal_host(200000, 0, 1, 1.0)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1.0) < 0.01 and np.abs(x).max() <= 6.0
    w = synth.mxfp4_host(50000, 0, 2).reshape(-1, 17)
    scales = w[:, 0]
    assert scales.min() == 119 and scales.max() == 125  # exponent -8..-2
    nib = np.concatenate([w[:, 1:] & 15, w[:, 1:] >> 4]).ravel()
    counts = np.bincount(nib, minlength=16)
    assert counts.min() > 0.95 * counts.mean() and counts.max() < 1.05 * counts.mean()


def test_zipf_shift_skews_routing():
    from ttl_moe import synth
    s = synth.zipf_shift(0, 32, 1.1)
    assert s.shape == (32,) and np.isclose(np.log(np.exp(s).sum()), 0.0, atol=1e-5)
    order = np.argsort(-s)
    assert len(set(order[:4])) == 4


def test_oracle_generator_matches_library():
    """The checker's own generator (oracle/synth_oracle.c) gives the library's
    tensors bit for bit, so the CPU side never needs the product library."""
    from oracle import synth as osynth
    from ttl_moe import synth
    a = osynth.layer_host(2, 3, 32, zipf_s=1.1, norm=True)
    b = synth.layer_host(2, 3, 32, zipf_s=1.1, norm=True)
    assert a.keys() == b.keys()
    for k in a:
        assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
    assert np.array_equal(osynth.inputs_host(5, 9).view(np.uint32), synth.inputs_host(5, 9).view(np.uint32))
    # block ranges split over threads give the single-range bytes
    one = osynth.mxfp4_host(300000, 7, 4, threads=1)
    many = osynth.mxfp4_host(300000, 7, 4, threads=5)
    assert np.array_equal(one, many)
