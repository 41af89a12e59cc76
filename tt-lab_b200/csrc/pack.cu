// pack.cu -- GPU weight-layout packer (requant) and the synthetic-input fillers.
//
// The packer replaces tt-lab's Tensix BFP8 strip payload (write_bfp8_strip_payload,
// src/requant.cpp:258-277) with a lossless re-layout of the GGUF MXFP4 blocks
// (src/tensor.cpp:116-131 reads block [scale][16 quant bytes]; byte i holds
// element i in the low nibble and element i+16 in the high nibble):
//   nibbles: element k of a row in byte k/2, low nibble for even k, rows of
//            1440 bytes -- the packed-FP4 row-major order that 16-byte vector
//            loads and TMA tiles stream directly;
//   scales:  the row's 90 E8M0 bytes split out into a 96-byte row (zero pad).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "synth.h"

namespace ttl {
namespace {

// One thread per (matrix, row, block).
// flags (optional): bit 0 is set when a scale byte is 255 -- tt-lab reads it as
// 2^128 (src/tensor.cpp:36-44), which has no E8M0 encoding for the tensor cores.
__global__ void pack_kernel(const uint8_t *__restrict__ gguf, uint8_t *__restrict__ packed, size_t blocks,
                            uint32_t *flags = nullptr) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < blocks; i += size_t(gridDim.x) * blockDim.x) {
        const size_t row_all = i / kBlocks;
        const int b = int(i % kBlocks);
        const size_t m = row_all / kDim;
        const size_t r = row_all % kDim;
        const uint8_t *src = gguf + i * 17;
        uint8_t q[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            q[j] = src[1 + j];
        }
        uint32_t w[4];
#pragma unroll
        for (int word = 0; word < 4; ++word) {
            uint32_t v = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int j = word * 4 + k;
                uint32_t byte;
                if (j < 8) {
                    byte = (q[2 * j] & 0x0fu) | ((q[2 * j + 1] & 0x0fu) << 4);
                } else {
                    byte = (q[2 * j - 16] >> 4) | (q[2 * j - 15] & 0xf0u);
                }
                v |= byte << (8 * k);
            }
            w[word] = v;
        }
        uint8_t *base = packed + m * kPackedMatrixBytes;
        *reinterpret_cast<uint4 *>(base + r * kNibbleRowBytes + size_t(b) * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        base[scale_offset(int(r), b)] = src[0];
        if (flags && src[0] == 255u) {
            atomicOr(flags, 1u);
        }
    }
}

__global__ void unpack_kernel(const uint8_t *__restrict__ packed, uint8_t *__restrict__ gguf, size_t blocks) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < blocks; i += size_t(gridDim.x) * blockDim.x) {
        const size_t row_all = i / kBlocks;
        const int b = int(i % kBlocks);
        const size_t m = row_all / kDim;
        const size_t r = row_all % kDim;
        const uint8_t *base = packed + m * kPackedMatrixBytes;
        const uint4 v = *reinterpret_cast<const uint4 *>(base + r * kNibbleRowBytes + size_t(b) * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint8_t e[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t byte = (w[j >> 2] >> (8 * (j & 3))) & 0xffu;
            e[2 * j] = uint8_t(byte & 0x0fu);
            e[2 * j + 1] = uint8_t(byte >> 4);
        }
        uint8_t *dst = gguf + i * 17;
        dst[0] = base[scale_offset(int(r), b)];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            dst[1 + j] = uint8_t(e[j] | (e[j + 16] << 4));
        }
    }
}

__global__ void scan_scales_kernel(const uint8_t *packed, size_t matrices, uint32_t *flags) {
    const size_t per = kPackedMatrixBytes - kNibbleBytes;  // the scale region of a matrix
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < matrices * per;
         i += size_t(gridDim.x) * blockDim.x) {
        const size_t m = i / per;
        if (packed[m * kPackedMatrixBytes + kNibbleBytes + (i - m * per)] == 255u) {
            atomicOr(flags, 1u);
        }
    }
}

__global__ void synth_mxfp4_kernel(uint8_t *dst, size_t blocks, uint64_t key, uint32_t lo, uint32_t count) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < blocks; i += size_t(gridDim.x) * blockDim.x) {
        uint8_t *out = dst + i * 17;
        for (uint32_t o = 0; o < 17; ++o) {
            out[o] = ttl_synth_mxfp4_byte(key, i, o, lo, count);
        }
    }
}

__global__ void synth_q8_0_kernel(uint8_t *dst, size_t blocks, uint64_t key) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < blocks; i += size_t(gridDim.x) * blockDim.x) {
        uint8_t *out = dst + i * 34;
        for (uint32_t o = 0; o < 34; ++o) {
            out[o] = ttl_synth_q8_0_byte(key, i, o);
        }
    }
}

__global__ void synth_normal_kernel(float *dst, size_t n, uint64_t key, float sigma, float mean) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        dst[i] = __fadd_rn(__fmul_rn(ttl_synth_normal(key, i), sigma), mean);
    }
}

int grid_for(size_t n) {
    return int(std::min<size_t>((n + 255) / 256, 148 * 32));
}

int select_device(int device) {
    if (device >= 0) {
        return int(cudaSetDevice(device));
    }
    return 0;
}

} // namespace
} // namespace ttl

using namespace ttl;

extern "C" size_t ttl_packed_bytes(size_t matrices) {
    return matrices * kPackedMatrixBytes;
}

namespace {

// Runs `kernel` over `matrices` matrices, staging host buffers through the
// device in chunks when either side is host memory.
template <class Kernel>
int run_repack(const void *src, size_t src_matrix_bytes, void *dst, size_t dst_matrix_bytes, size_t matrices,
               int device, Kernel kernel) {
    if ((!src || !dst) && matrices) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null buffer");
    }
    if (select_device(device) != 0) {
        return fail(nullptr, TTL_ERR_CUDA, "cannot select device");
    }
    const bool src_dev = is_device_pointer(src);
    const bool dst_dev = is_device_pointer(dst);
    const size_t chunk = (src_dev && dst_dev) ? std::max<size_t>(matrices, 1) : 16;
    uint8_t *dsrc = nullptr;
    uint8_t *ddst = nullptr;
    int rc = TTL_OK;
    if (!src_dev && cudaMalloc(&dsrc, chunk * src_matrix_bytes) != cudaSuccess) {
        return fail(nullptr, TTL_ERR_CUDA, "cannot allocate packer staging buffer");
    }
    if (!dst_dev && cudaMalloc(&ddst, chunk * dst_matrix_bytes) != cudaSuccess) {
        cudaFree(dsrc);
        return fail(nullptr, TTL_ERR_CUDA, "cannot allocate packer staging buffer");
    }
    for (size_t m0 = 0; m0 < matrices && rc == TTL_OK; m0 += chunk) {
        const size_t n = std::min(chunk, matrices - m0);
        const uint8_t *s = (const uint8_t *)src + m0 * src_matrix_bytes;
        uint8_t *d = (uint8_t *)dst + m0 * dst_matrix_bytes;
        if (!src_dev) {
            if (cudaMemcpy(dsrc, s, n * src_matrix_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
                rc = fail(nullptr, TTL_ERR_CUDA, "packer upload failed");
                break;
            }
            s = dsrc;
        }
        uint8_t *out = dst_dev ? d : ddst;
        const size_t blocks = n * size_t(kDim) * kBlocks;
        kernel(s, out, blocks);
        if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            rc = fail(nullptr, TTL_ERR_CUDA, "packer kernel failed");
            break;
        }
        if (!dst_dev && cudaMemcpy(d, ddst, n * dst_matrix_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
            rc = fail(nullptr, TTL_ERR_CUDA, "packer download failed");
        }
    }
    cudaFree(dsrc);
    cudaFree(ddst);
    return rc;
}

} // namespace

extern "C" int ttl_pack_mxfp4(const void *gguf, size_t matrices, void *packed, int device) {
    const size_t gguf_bytes = size_t(kDim) * kGgufRowBytes;
    return run_repack(gguf, gguf_bytes, packed, kPackedMatrixBytes, matrices, device,
                      [](const uint8_t *s, uint8_t *d, size_t blocks) {
                          cudaMemset2DAsync(d + kNibbleBytes, kPackedMatrixBytes, 0, kScaleBytes,
                                            blocks / (size_t(kDim) * kBlocks), 0);
                          pack_kernel<<<grid_for(blocks), 256>>>(s, d, blocks);
                      });
}

extern "C" int ttl_unpack_mxfp4(const void *packed, size_t matrices, void *gguf, int device) {
    const size_t gguf_bytes = size_t(kDim) * kGgufRowBytes;
    return run_repack(packed, kPackedMatrixBytes, gguf, gguf_bytes, matrices, device,
                      [](const uint8_t *s, uint8_t *d, size_t blocks) {
                          unpack_kernel<<<grid_for(blocks), 256>>>(s, d, blocks);
                      });
}

// Device-side packing used by ttl_moe_upload_layer (stream-ordered, no sync).
namespace ttl {
void launch_pack(const uint8_t *gguf_dev, uint8_t *packed_dev, size_t matrices, cudaStream_t stream,
                 uint32_t *flags) {
    const size_t blocks = matrices * size_t(kDim) * kBlocks;
    if (blocks) {
        // scale padding (K-blocks 90, 91; rows 2880..2943; the region's tail) is zero
        cudaMemset2DAsync(packed_dev + kNibbleBytes, kPackedMatrixBytes, 0, kScaleBytes, matrices, stream);
        pack_kernel<<<grid_for(blocks), 256, 0, stream>>>(gguf_dev, packed_dev, blocks, flags);
    }
}
} // namespace ttl

namespace ttl {
void launch_scan_scales(const uint8_t *packed_dev, size_t matrices, cudaStream_t stream, uint32_t *flags) {
    const size_t n = matrices * (kPackedMatrixBytes - kNibbleBytes);
    if (n) {
        scan_scales_kernel<<<grid_for(n), 256, 0, stream>>>(packed_dev, matrices, flags);
    }
}
} // namespace ttl

extern "C" int ttl_synth_mxfp4(void *dst, size_t blocks, uint64_t seed, uint64_t stream, uint32_t scale_lo,
                               uint32_t scale_count) {
    if (!dst && blocks) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null buffer");
    }
    if (scale_count == 0 || scale_lo + scale_count > 256) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "scale range outside 0..255");
    }
    const uint64_t key = ttl_synth_key(seed, stream);
    if (is_device_pointer(dst)) {
        synth_mxfp4_kernel<<<grid_for(blocks), 256>>>((uint8_t *)dst, blocks, key, scale_lo, scale_count);
        TTL_TRY_CUDA(nullptr, cudaGetLastError());
        TTL_TRY_CUDA(nullptr, cudaDeviceSynchronize());
        return TTL_OK;
    }
    // Same bytes as ttl_synth_mxfp4_byte, three draws per block.
    uint8_t *out = (uint8_t *)dst;
    for (size_t i = 0; i < blocks; ++i) {
        const uint64_t h0 = ttl_synth_draw(key, i * 3ull);
        const uint64_t h1 = ttl_synth_draw(key, i * 3ull + 1ull);
        const uint64_t h2 = ttl_synth_draw(key, i * 3ull + 2ull);
        uint8_t *b = out + i * 17;
        b[0] = (uint8_t)(scale_lo + (uint32_t)(((h2 >> 32) * (uint64_t)scale_count) >> 32));
        for (int q = 0; q < 8; ++q) {
            b[1 + q] = (uint8_t)(h0 >> (8 * q));
            b[9 + q] = (uint8_t)(h1 >> (8 * q));
        }
    }
    return TTL_OK;
}

extern "C" int ttl_synth_q8_0(void *dst, size_t blocks, uint64_t seed, uint64_t stream) {
    if (!dst && blocks) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null buffer");
    }
    const uint64_t key = ttl_synth_key(seed, stream);
    if (is_device_pointer(dst)) {
        synth_q8_0_kernel<<<grid_for(blocks), 256>>>((uint8_t *)dst, blocks, key);
        TTL_TRY_CUDA(nullptr, cudaGetLastError());
        TTL_TRY_CUDA(nullptr, cudaDeviceSynchronize());
        return TTL_OK;
    }
    uint8_t *out = (uint8_t *)dst;
    for (size_t i = 0; i < blocks; ++i) {
        for (uint32_t o = 0; o < 34; ++o) {
            out[i * 34 + o] = ttl_synth_q8_0_byte(key, i, o);
        }
    }
    return TTL_OK;
}

extern "C" int ttl_synth_normal(float *dst, size_t n, uint64_t seed, uint64_t stream, float sigma, float mean) {
    if (!dst && n) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null buffer");
    }
    const uint64_t key = ttl_synth_key(seed, stream);
    if (is_device_pointer(dst)) {
        synth_normal_kernel<<<grid_for(n), 256>>>(dst, n, key, sigma, mean);
        TTL_TRY_CUDA(nullptr, cudaGetLastError());
        TTL_TRY_CUDA(nullptr, cudaDeviceSynchronize());
        return TTL_OK;
    }
    for (size_t i = 0; i < n; ++i) {
        // Two separately rounded IEEE operations, as in the kernel.
        volatile float scaled = ttl_synth_normal(key, i) * sigma;
        dst[i] = scaled + mean;
    }
    return TTL_OK;
}
