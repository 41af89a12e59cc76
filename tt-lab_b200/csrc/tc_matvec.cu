// tc_matvec.cu -- one 2880 x 2880 MXFP4 expert matrix times an f32 vector on
// the tcgen05 tensor cores: y = bias + W x, tt-lab's matvec_add_mxfp4_2880
// (src/tensor.cpp:239-304).
//
// One CTA per 128-row tile (23 tiles, the last one half used).  The packed
// E2M1 nibbles are copied into shared memory as 8-byte runs into 16-byte slots
// (the layout the block-scaled MXF8F6F4 MMA reads for FP4 operands), the
// row scales go to tensor memory, x is split into four E4M3 terms (B, N = 8),
// and 90 MMAs of K = 32 accumulate the tile in tensor memory.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace ttl {
namespace {

constexpr int kTerms = 4;
constexpr int kN = 8;                           // MMA N (terms padded to 8)
constexpr int kChunks = kDim / 16;              // 180 16-element K-chunks
constexpr int kStageBlocks = 4;                 // K-blocks per stage (one SF chunk)
constexpr int kStageChunks = kStageBlocks * 2;  // 8 K-chunks of 16 elements
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kColD = 0;                   // D: 8 columns
constexpr uint32_t kColSfb = 8;                 // SFB: 23 chunks x 4 columns
constexpr uint32_t kColSfa = 100;               // SFA: 4 columns (one stage)

struct MatvecSmem {
    alignas(128) uint8_t b[kChunks][kN][16];                  // B terms, K-major core matrices
    alignas(128) uint8_t a[16][kStageChunks][8][16];          // A stage: [row group][chunk][row][16 B]
    uint8_t sfb[kBlocks][kTerms];                             // term scales per K-block
    alignas(8) uint64_t bar;
    uint32_t tmem;
    int failed;
};

__global__ void __launch_bounds__(128, 1)
    tc_matvec_kernel(const uint8_t *__restrict__ packed, const float *__restrict__ bias,
                     const float *__restrict__ x, float *__restrict__ y, uint32_t *status) {
    extern __shared__ __align__(128) unsigned char raw[];
    MatvecSmem &s = *reinterpret_cast<MatvecSmem *>(raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * 128;

    if (warp == 0) {
        tc::tmem_alloc(&s.tmem, kTmemCols);
        tc::tmem_relinquish();
    }
    if (threadIdx.x == 0) {
        tc::mbar_init(&s.bar, 1);
        tc::fence_mbar_init();
        s.failed = 0;
    }
    // B: x split into terms; row n of B is term n (rows 4..7 zero).
    for (int kb = warp; kb < kBlocks; kb += 4) {
        uint32_t sc;
        const uint32_t t = tc::split_terms<kTerms>(x[kb * 32 + lane], sc);
        const int k = kb * 32 + lane;
#pragma unroll
        for (int n = 0; n < kN; ++n) {
            s.b[k >> 4][n][k & 15] = n < kTerms ? uint8_t(t >> (8 * n)) : uint8_t(0);
        }
        if (lane == 0) {
#pragma unroll
            for (int n = 0; n < kTerms; ++n) {
                s.sfb[kb][n] = uint8_t(sc >> (8 * n));
            }
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = s.tmem;
    const uint32_t lane_base = uint32_t(warp * 32) << 16;

    // SFB: chunk g -> column kColSfb + 4g, lane n (< 4) holds term n's 4 bytes.
    for (int g = 0; g < (kBlocks + 3) / 4; ++g) {
        uint32_t v = 0;
        if (lane < kTerms) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int kb = 4 * g + k;
                v |= (kb < kBlocks ? uint32_t(s.sfb[kb][lane]) : 127u) << (8 * k);
            }
        }
        tc::tmem_st4(tbase + lane_base + kColSfb + 4 * g, v, 0u, 0u, 0u);
    }

    const uint32_t idesc0 = tc::instr_desc(kN, 0, 0);
    uint32_t phase = 0;
    for (int kb0 = 0; kb0 < kBlocks; kb0 += kStageBlocks) {
        const int nkb = min(kStageBlocks, kBlocks - kb0);
        // A stage: 128 rows x nkb K-blocks, 8 packed bytes per 16-byte slot.
        for (int i = threadIdx.x; i < 128 * kStageChunks; i += 128) {
            const int row = i / kStageChunks;
            const int c = i % kStageChunks;
            const int r = r0 + row;
            if (r < kDim && c < 2 * nkb) {
                const uint8_t *src = packed + size_t(r) * kNibbleRowBytes + size_t(kb0) * 16 + c * 8;
                asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(tc::smem_u32(&s.a[row >> 3][c][row & 7][0])),
                             "l"(src)
                             : "memory");
            }
        }
        // SFA: warp q, thread m0 -> columns kColSfa..+3 = rows m0 + 32*m1.
        {
            uint32_t v[4];
#pragma unroll
            for (int m1 = 0; m1 < 4; ++m1) {
                const int r = r0 + lane + 32 * m1;
                v[m1] = 0;
                if (r < kDim) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        v[m1] |= uint32_t(packed[scale_offset(r, kb0 + k)]) << (8 * k);
                    }
                }
            }
            tc::tmem_st4(tbase + lane_base + kColSfa, v[0], v[1], v[2], v[3]);
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc::wait_st();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (threadIdx.x == 0) {
            const uint32_t a_base = tc::smem_u32(&s.a[0][0][0][0]);
            const uint32_t b_base = tc::smem_u32(&s.b[0][0][0]);
            for (int j = 0; j < nkb; ++j) {
                const int kb = kb0 + j;
                const uint64_t ad = tc::smem_desc(a_base + uint32_t(j) * 2 * 128, 128, kStageChunks * 128);
                const uint64_t bd = tc::smem_desc(b_base + uint32_t(kb) * 2 * 128, 128, kChunks * 128);
                const uint32_t idesc = idesc0 | (uint32_t(kb & 3) << 4) | (uint32_t(j) << 29);
                const uint32_t sfa = (tbase + kColSfa) | (uint32_t(j) << 30);
                const uint32_t sfb = (tbase + kColSfb + 4 * (kb >> 2)) | (uint32_t(kb & 3) << 30);
                tc::mma(tbase + kColD, ad, bd, idesc, sfa, sfb, kb > 0);
            }
            tc::mma_commit(&s.bar);
        }
        __syncwarp();
        // the stage buffers are reused: wait for the MMAs reading them
        if (!tc::mbar_wait(&s.bar, phase)) {
            if (lane == 0) {
                set_status(status, kStatusWaitTimeout);
            }
            s.failed = 1;
        }
        phase ^= 1u;
        tc::fence_after_sync();
        __syncthreads();
        if (s.failed) {
            break;
        }
    }
    if (!s.failed) {
        float d[8];
        tc::tmem_ld8(tbase + lane_base + kColD, d);
        tc::wait_ld();
        const int r = r0 + warp * 32 + lane;
        if (r < kDim) {
            float acc = 0.0f;
#pragma unroll
            for (int n = 0; n < kTerms; ++n) {
                acc += d[n];
            }
            y[r] = __fadd_rn(bias[r], acc);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
}

} // namespace
} // namespace ttl

using namespace ttl;

extern "C" int ttl_matvec_mxfp4(const void *packed, const float *bias, const float *x, float *y, int device) {
    if (!packed || !bias || !x || !y) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null pointer");
    }
    if (device >= 0 && cudaSetDevice(device) != cudaSuccess) {
        return fail(nullptr, TTL_ERR_CUDA, "cannot select device");
    }
    if (!is_device_pointer(packed) || !is_device_pointer(bias) || !is_device_pointer(x) || !is_device_pointer(y)) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "ttl_matvec_mxfp4 takes device pointers");
    }
    uint32_t *status = nullptr;
    TTL_TRY_CUDA(nullptr, cudaMalloc(&status, sizeof(uint32_t)));
    const int smem = int(sizeof(MatvecSmem));
    cudaError_t e = cudaMemset(status, 0, sizeof(uint32_t));
    if (e == cudaSuccess) {
        e = cudaFuncSetAttribute(tc_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    }
    if (e == cudaSuccess) {
        tc_matvec_kernel<<<(kDim + 127) / 128, 128, smem>>>((const uint8_t *)packed, bias, x, y, status);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        e = cudaDeviceSynchronize();
    }
    uint32_t st = 0;
    if (e == cudaSuccess) {
        e = cudaMemcpy(&st, status, sizeof(st), cudaMemcpyDeviceToHost);
    }
    cudaFree(status);
    if (e != cudaSuccess) {
        return fail(nullptr, TTL_ERR_CUDA, std::string("tc matvec: ") + cudaGetErrorString(e));
    }
    if (st) {
        return fail(nullptr, TTL_ERR_DEVICE, "tc matvec: bounded wait gave up");
    }
    return TTL_OK;
}

// ---- allocation-free variant ----
// Status words of ttl_matvec_mxfp4_noalloc live in this file-scope array
// instead of a per-call cudaMalloc: one word per matrix of a call.  The
// array's device address is looked up once per device ordinal and kept for
// the life of the process, so a device reset (cudaDeviceReset, or a context
// torn down and made again) is not supported for callers of this entry.
namespace {
constexpr size_t kNoAllocMaxMatrices = 256;  // 1 KB of scratch per device
static __device__ __align__(256) uint32_t g_noalloc_status[kNoAllocMaxMatrices];

std::mutex g_noalloc_mutex;
void *g_noalloc_addr[64] = {};  // per device ordinal, looked up once
} // namespace

extern "C" int ttl_matvec_mxfp4_noalloc(const void *packed, const float *bias, const float *x, float *y,
                                        size_t matrices, int device) {
    if (!packed || !bias || !x || !y) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null pointer");
    }
    if (matrices == 0 || matrices > kNoAllocMaxMatrices) {
        return fail(nullptr, TTL_ERR_ARGUMENT,
                    "ttl_matvec_mxfp4_noalloc takes 1.." + std::to_string(kNoAllocMaxMatrices) +
                        " matrices per call (its scratch is a fixed static array); got " + std::to_string(matrices));
    }
    if (device >= 0 && cudaSetDevice(device) != cudaSuccess) {
        return fail(nullptr, TTL_ERR_CUDA, "cannot select device");
    }
    int dev = 0;
    TTL_TRY_CUDA(nullptr, cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) {
        return fail(nullptr, TTL_ERR_UNSUPPORTED, "device ordinal above 63");
    }
    if (!is_device_pointer(packed) || !is_device_pointer(bias) || !is_device_pointer(x) || !is_device_pointer(y)) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "ttl_matvec_mxfp4_noalloc takes device pointers");
    }
    uint32_t *status = nullptr;
    {
        // first call on this device: look the scratch up (and set the kernel's
        // shared-memory limit) with the device current
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if (!g_noalloc_addr[dev]) {
            void *addr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_status);
            if (e != cudaSuccess || !addr) {
                return fail(nullptr, TTL_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            }
            TTL_TRY_CUDA(nullptr, cudaFuncSetAttribute(tc_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       int(sizeof(MatvecSmem))));
            g_noalloc_addr[dev] = addr;
        }
        status = static_cast<uint32_t *>(g_noalloc_addr[dev]);
    }
    // the status words start at zero
    TTL_TRY_CUDA(nullptr, cudaMemsetAsync(status, 0, matrices * sizeof(uint32_t), 0));
    for (size_t m = 0; m < matrices; ++m) {
        tc_matvec_kernel<<<(kDim + 127) / 128, 128, int(sizeof(MatvecSmem))>>>(
            static_cast<const uint8_t *>(packed) + m * kPackedMatrixBytes, bias + m * kDim, x + m * kDim, y + m * kDim,
            status + m);
    }
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
        e = cudaStreamSynchronize(0);
    }
    uint32_t st[kNoAllocMaxMatrices];
    if (e == cudaSuccess) {
        e = cudaMemcpy(st, status, matrices * sizeof(uint32_t), cudaMemcpyDeviceToHost);
    }
    if (e != cudaSuccess) {
        return fail(nullptr, TTL_ERR_CUDA, std::string("tc matvec: ") + cudaGetErrorString(e));
    }
    for (size_t m = 0; m < matrices; ++m) {
        if (st[m]) {
            return fail(nullptr, TTL_ERR_DEVICE, "tc matvec: bounded wait gave up on matrix " + std::to_string(m));
        }
    }
    return TTL_OK;
}
