// common.cuh -- constants and device helpers shared by the MoE kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ttl {

constexpr int kDim = 2880;            // hidden = expert intermediate (tt-lab src/model.h:34, :43)
constexpr int kBlocks = kDim / 32;    // 90 MXFP4 blocks per row (src/tensor.cpp:78)
constexpr int kGgufRowBytes = kBlocks * 17;  // 1530 (src/tensor.cpp:79)
constexpr int kTopK = 4;              // src/model.h:42
constexpr int kMaxExperts = 128;      // src/model.h:41

// Packed GPU layout of one 2880 x 2880 MXFP4 matrix (TTQ format 6):
//   nibbles: [2880 rows][1440 B]; element k of a row sits in byte k/2, low
//            nibble for even k (the order TMA and the tensor cores use);
//   scales:  the E8M0 block scales, tile-blocked: for each 128-row tile t (23;
//            rows past 2879 are zero) and each chunk c of 4 K-blocks (23;
//            K-blocks 90 and 91 are zero), one 512-byte block ordered
//            [row % 32][(row % 128) / 32][K-block % 4] -- the order in which
//            tcgen05.cp moves an M = 128 tile's scales into tensor memory, so
//            a tile's scales for 4 K-blocks are one contiguous copy.  Blocks
//            are stored tile-major ((t * 23 + c) * 512); the region is padded
//            with zeros to 2880 x 96 bytes.
constexpr int kNibbleRowBytes = kDim / 2;   // 1440
constexpr size_t kNibbleBytes = size_t(kDim) * kNibbleRowBytes;  // 4,147,200
constexpr size_t kScaleBytes = size_t(kDim) * 96;                // 276,480
constexpr size_t kPackedMatrixBytes = kNibbleBytes + kScaleBytes;  // 4,423,680
constexpr int kScaleTiles = (kDim + 127) / 128;  // 23
constexpr int kScaleChunks = (kBlocks + 3) / 4;  // 23
constexpr size_t kScaleBlockBytes = 512;
static_assert(size_t(kScaleTiles) * kScaleChunks * kScaleBlockBytes <= kScaleBytes, "scale layout");

// Byte offset, from the start of a packed matrix, of the scale of (row, K-block).
__host__ __device__ __forceinline__ constexpr size_t scale_offset(int row, int kb) {
    return kNibbleBytes + (size_t(row >> 7) * kScaleChunks + size_t(kb >> 2)) * kScaleBlockBytes +
           size_t(row & 31) * 16 + size_t((row >> 5) & 3) * 4 + size_t(kb & 3);
}

// Offset of the 512-byte scale block of (128-row tile, 4-K-block chunk).
__host__ __device__ __forceinline__ constexpr size_t scale_block_offset(int tile, int chunk) {
    return kNibbleBytes + (size_t(tile) * kScaleChunks + size_t(chunk)) * kScaleBlockBytes;
}

// Device status word bits (set by kernels, read by ttl_moe_sync).
enum : uint32_t {
    kStatusBadExpert = 1u << 0,     // an expert index outside [0, E)
    kStatusCapacity = 1u << 1,      // a token count above the buffers' capacity
    kStatusWaitTimeout = 1u << 2,   // a bounded wait gave up
    kStatusBadShape = 1u << 3,
};

__device__ __forceinline__ void set_status(uint32_t *status, uint32_t bit) {
    atomicOr(status, bit);
}

// E8M0 byte -> 2^(e-128), the reference's mxfp4_scale (src/tensor.cpp:36-44):
// denormal for e < 2, 2^127 for e == 255.  The reference multiplies it by the
// doubled E2M1 table (src/tensor.cpp:34); the kernels multiply it by twice the
// exact E2M1 block partial, which is the same value.
__device__ __forceinline__ float e8m0_ref_scale(uint32_t e) {
    return e < 2 ? __uint_as_float(0x00200000u << e) : __uint_as_float((e - 1u) << 23);
}

// Two E2M1 codes (low nibble = first element) -> two exact f16 values.
__device__ __forceinline__ __half2 e2m1x2_to_half2(uint32_t byte) {
    uint32_t out;
    asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(out) : "r"(byte));
    return *reinterpret_cast<__half2 *>(&out);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    return v;
}

// Clamped SwiGLU of tt-lab src/model.cpp:328-332 with IEEE operations in the
// reference's order (no contraction): min(gate, 7), clamp(up, -7, 7),
// (x / (1 + exp(-1.702 x))) * (y + 1).
__device__ __forceinline__ float swiglu_ref(float gate, float up) {
    const float x = (7.0f < gate) ? 7.0f : gate;
    const float y = (up < -7.0f) ? -7.0f : ((7.0f < up) ? 7.0f : up);
    const float t = __fmul_rn(-1.702f, x);
    const float d = __fadd_rn(1.0f, expf(t));
    const float q = __fdiv_rn(x, d);
    return __fmul_rn(q, __fadd_rn(y, 1.0f));
}

} // namespace ttl
