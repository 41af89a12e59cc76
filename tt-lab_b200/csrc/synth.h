// synth.h -- seeded synthetic gpt-oss MoE inputs, bit-identical on host and device.
//
// The real gpt-oss GGUF files are not available to the tests or the benchmark, so
// weights and activations are generated from (seed, stream, index) with a
// counter-based hash (the SplitMix64 finaliser over seed-dependent counters).
// Every value depends only on integer arithmetic, so the host and the device
// produce the same bits and the CPU reference sees exactly the GPU's inputs:
//
//   - MXFP4 expert tensors in GGUF layout (17-byte blocks, src/tensor.cpp:76-79
//     and :149-153 of tt-lab): 16 quant bytes uniform over 0..255 (so both
//     nibbles are uniform over the 16 E2M1 codes) and one E8M0 scale byte
//     uniform over [scale_lo, scale_lo + scale_count).
//   - Q8_0 tensors in GGUF layout (34-byte blocks, src/tensor.cpp:90-114): a
//     half scale with bits 0x1000 + 11 random bits (2^-11 <= scale < 2^-9,
//     the range of a gpt-oss output matrix), then 32 int8 quants uniform over
//     -128..127 (five draws per block).
//   - "Normal" f32 values: Irwin-Hall with twelve 24-bit uniforms,
//     sum - 6 (mean 0, variance 1, bounded by +-6), times sigma.  The sum is
//     formed in integers and converted once, so it rounds identically everywhere.
#pragma once

#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define TTL_HD __host__ __device__ __forceinline__
#else
#define TTL_HD static inline
#endif

TTL_HD uint64_t ttl_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Key of one stream (one tensor) for a seed.
TTL_HD uint64_t ttl_synth_key(uint64_t seed, uint64_t stream) {
    return ttl_mix64(ttl_mix64(seed + 0x9E3779B97F4A7C15ull) ^ (stream * 0xD1B54A32D192ED03ull + 1ull));
}

// i-th 64-bit draw of a stream.
TTL_HD uint64_t ttl_synth_draw(uint64_t key, uint64_t i) {
    return ttl_mix64(key + (i + 1ull) * 0x9E3779B97F4A7C15ull);
}

// i-th approximately N(0,1) value of a stream (Irwin-Hall of 12 uniforms).
TTL_HD float ttl_synth_normal(uint64_t key, uint64_t i) {
    int64_t sum = 0;
    for (uint64_t j = 0; j < 6; ++j) {
        const uint64_t h = ttl_synth_draw(key, i * 6ull + j);
        sum += (int64_t)(h & 0xFFFFFFull) + (int64_t)((h >> 32) & 0xFFFFFFull);
    }
    const int32_t centred = (int32_t)(sum - 100663296ll); // 6 * 2^24
    return (float)centred * 5.9604644775390625e-08f;      // * 2^-24, exact
}

// Byte `offset` of block `block` of an MXFP4 tensor in GGUF layout.
TTL_HD uint8_t ttl_synth_mxfp4_byte(uint64_t key, uint64_t block, uint32_t offset, uint32_t scale_lo,
                                    uint32_t scale_count) {
    if (offset == 0) {
        const uint64_t h = ttl_synth_draw(key, block * 3ull + 2ull);
        return (uint8_t)(scale_lo + (uint32_t)(((h >> 32) * (uint64_t)scale_count) >> 32));
    }
    const uint32_t q = offset - 1;
    const uint64_t h = ttl_synth_draw(key, block * 3ull + (q >> 3));
    return (uint8_t)(h >> (8 * (q & 7)));
}

// Byte `offset` (0..33) of block `block` of a Q8_0 tensor in GGUF layout.
TTL_HD uint8_t ttl_synth_q8_0_byte(uint64_t key, uint64_t block, uint32_t offset) {
    if (offset < 2) {
        const uint64_t h = ttl_synth_draw(key, block * 5ull + 4ull);
        const uint32_t bits = 0x1000u + (uint32_t)((h >> 40) & 0x7FFull);
        return (uint8_t)(bits >> (8 * offset));
    }
    const uint32_t q = offset - 2;
    const uint64_t h = ttl_synth_draw(key, block * 5ull + (q >> 3));
    return (uint8_t)(h >> (8 * (q & 7)));
}
