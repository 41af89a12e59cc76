/*
 * synth_oracle.c -- the benchmark's seeded synthetic inputs, generated on the
 * CPU for the checker and for the reference arm of the benchmark.
 *
 * TEST INFRASTRUCTURE ONLY.  The product library has its own generator for
 * device-resident inputs; this is an independent restatement of the same
 * counter-based definition, so that the CPU side (the oracle, tt-lab's
 * compiled code in oracle/_ref, and bench.py --impl reference) never needs the
 * product library to make its inputs.  tests/test_synth.py holds the two
 * generators to the same bits.
 *
 * Definition (all integer arithmetic, identical on every machine):
 *   mix(z)       the SplitMix64 finaliser (Steele, Lea, Flood 2014):
 *                z ^= z >> 30; z *= 0xBF58476D1CE4E5B9; z ^= z >> 27;
 *                z *= 0x94D049BB133111EB; z ^= z >> 31
 *   key(s, t)    mix(mix(s + golden) ^ (t * 0xD1B54A32D192ED03 + 1)), golden =
 *                0x9E3779B97F4A7C15, for seed s and stream t (one per tensor)
 *   draw(k, i)   mix(k + (i + 1) * golden)
 *   normal(k, i) (sum over j < 6 of the low and high 24-bit fields of
 *                draw(k, 6i + j)) - 6 * 2^24, times 2^-24: Irwin-Hall of 12
 *                uniforms, mean 0, variance 1, formed in integers
 *   MXFP4 block b (GGUF layout, 17 bytes): byte 0 = lo + ((hi32(draw(k, 3b + 2))
 *                * count) >> 32); bytes 1..8 and 9..16 = the little-endian bytes
 *                of draw(k, 3b) and draw(k, 3b + 1)
 *   Q8_0 block b (GGUF layout, 34 bytes): bytes 0..1 = the half bits 0x1000 +
 *                ((draw(k, 5b + 4) >> 40) & 0x7FF), little-endian; bytes 2..33 =
 *                the little-endian bytes of draw(k, 5b) .. draw(k, 5b + 3)
 */
#include <stddef.h>
#include <stdint.h>

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return mix64(mix64(seed + 0x9E3779B97F4A7C15ull) ^ (stream * 0xD1B54A32D192ED03ull + 1ull));
}

static inline uint64_t draw(uint64_t key, uint64_t i) {
    return mix64(key + (i + 1ull) * 0x9E3779B97F4A7C15ull);
}

/* Values i0 .. i0 + n - 1 of sigma * normal(key(seed, stream), i) + mean
 * (ranges let callers split a tensor over threads). */
void oref_synth_normal_range(float *dst, size_t i0, size_t n, uint64_t seed, uint64_t stream, float sigma,
                             float mean) {
    const uint64_t k = stream_key(seed, stream);
    for (size_t i = i0; i < i0 + n; ++i) {
        int64_t sum = 0;
        for (uint64_t j = 0; j < 6; ++j) {
            const uint64_t h = draw(k, (uint64_t)i * 6ull + j);
            sum += (int64_t)(h & 0xFFFFFFull) + (int64_t)((h >> 32) & 0xFFFFFFull);
        }
        const int32_t centred = (int32_t)(sum - 100663296ll);
        const float v = (float)centred * 5.9604644775390625e-08f;
        dst[i - i0] = v * sigma + mean;
    }
}

void oref_synth_normal(float *dst, size_t n, uint64_t seed, uint64_t stream, float sigma, float mean) {
    oref_synth_normal_range(dst, 0, n, seed, stream, sigma, mean);
}

/* GGUF MXFP4 blocks b0 .. b0 + blocks - 1; scale bytes uniform over
 * [lo, lo + count). */
void oref_synth_mxfp4_range(uint8_t *dst, size_t b0, size_t blocks, uint64_t seed, uint64_t stream, uint32_t lo,
                            uint32_t count) {
    const uint64_t k = stream_key(seed, stream);
    for (size_t b = b0; b < b0 + blocks; ++b) {
        uint8_t *o = dst + (b - b0) * 17;
        const uint64_t h0 = draw(k, (uint64_t)b * 3ull);
        const uint64_t h1 = draw(k, (uint64_t)b * 3ull + 1ull);
        const uint64_t h2 = draw(k, (uint64_t)b * 3ull + 2ull);
        o[0] = (uint8_t)(lo + (uint32_t)(((h2 >> 32) * (uint64_t)count) >> 32));
        for (int j = 0; j < 8; ++j) {
            o[1 + j] = (uint8_t)(h0 >> (8 * j));
            o[9 + j] = (uint8_t)(h1 >> (8 * j));
        }
    }
}

void oref_synth_mxfp4(uint8_t *dst, size_t blocks, uint64_t seed, uint64_t stream, uint32_t lo, uint32_t count) {
    oref_synth_mxfp4_range(dst, 0, blocks, seed, stream, lo, count);
}

/* GGUF Q8_0 blocks b0 .. b0 + blocks - 1. */
void oref_synth_q8_0_range(uint8_t *dst, size_t b0, size_t blocks, uint64_t seed, uint64_t stream) {
    const uint64_t k = stream_key(seed, stream);
    for (size_t b = b0; b < b0 + blocks; ++b) {
        uint8_t *o = dst + (b - b0) * 34;
        const uint64_t hs = draw(k, (uint64_t)b * 5ull + 4ull);
        const uint32_t bits = 0x1000u + (uint32_t)((hs >> 40) & 0x7FFull);
        o[0] = (uint8_t)bits;
        o[1] = (uint8_t)(bits >> 8);
        for (int d = 0; d < 4; ++d) {
            const uint64_t h = draw(k, (uint64_t)b * 5ull + (uint64_t)d);
            for (int j = 0; j < 8; ++j) {
                o[2 + 8 * d + j] = (uint8_t)(h >> (8 * j));
            }
        }
    }
}
