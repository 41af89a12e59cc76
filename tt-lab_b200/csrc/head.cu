// head.cu -- the output head of GptOssModel::forward / prefill on the GPU:
// normalized = rms_norm(x, output_norm.weight), logits = matvec_q8_0(
// output.weight, normalized), token = greedy(logits) (tt-lab
// src/model.cpp:598-612, src/tensor.cpp:202-218 and :568-580), bit for bit.
//
// Layout: at upload every GGUF Q8_0 row (90 blocks of a half scale and 32 int8
// quants, 3060 B) is repacked as [2880 quants][90 half scales][12 B zero], a
// 3072-byte row, so quants load as aligned 8-byte words.
//
// Arithmetic, the reference's exactly: per row, 32 independent chains -- chain
// j accumulates element j of every block in block order, each term rounded as
// (q * scale) * x and added with one rounding -- then acc[j] = chain j +
// chain j+16 for j < 16, and those 16 values summed in order from 0.0f.
// q * scale is exact (an 8-bit integer times an 11-bit significand); it is
// formed by one FMA from the float M whose second byte holds u = q + 128 above
// the exponent of 2^23: M = 2^23 + 256 u, so q * s = M (s / 256) - 32896 s with
// both products exact, and the FMA's single rounding of an exactly
// representable value changes nothing.
// rms_norm: the sum of squares is the reference's sequential f32 chain,
// scale = 1 / sqrt(sum / 2880 + 1e-5) with IEEE division and square root,
// normalized = (x * scale) * w.
//
// Kernel: head_kernel, one persistent CTA per SM.  A producer warp streams
// the CTA's stages (8 packed rows, 24 KB, one bulk copy per row) through an
// 8-deep shared-memory ring; two consumer warps per ring slot take four rows
// each, eight lanes per row, lane (row, sub) keeping the chains of elements
// 4 sub .. 4 sub + 3 (sub 0..3: elements 0..15, sub 4..7: 16..31).  Every
// CTA normalizes x itself, the chain on one thread while the first stages
// land.  The logits go out as they are made; the greedy argmax folds into one
// 64-bit atomicMax per CTA over keys (value order, -row), and the last CTA to
// finish decodes the token and re-arms the state.  Waits are bounded (2 s);
// a wait that gives up sets the status word the host reads.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace ttl {
namespace {

constexpr int kQ8Blocks = kDim / 32;             // 90
constexpr int kQ8RowBytes = kQ8Blocks * 34;      // 3060
constexpr int kPackedRowBytes = 3072;            // quants, scales, padding
constexpr int kStageRows = 8;
// Rows sit 3104 B apart in shared memory (one bulk copy per row): 3104 is 32
// B past a multiple of 128, so the four rows a warp reads together fall in
// different banks (at 3072 B they would all share each bank).
constexpr int kSmemRowStride = kPackedRowBytes + 32;
constexpr uint32_t kStageBytes = kStageRows * kSmemRowStride;  // 24,832
constexpr int kRing = 8;
constexpr int kConsumerWarps = 2 * kRing;        // two per ring slot, four rows each
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kHeadThreads = 32 * (kConsumerWarps + 1);
constexpr unsigned long long kHeadWaitNs = 2000000000ull;

// Device state of a head: the argmax key, the CTA arrival count, the flag for
// a NaN at row 0 and the token; the last CTA of a call re-arms the first three.
struct HeadState {
    unsigned long long key;
    unsigned int arrived;
    unsigned int nan0;
    int32_t token;
    uint32_t status;
};

struct alignas(1024) HeadSmem {
    uint8_t ring[kRing][kStageBytes];
    alignas(16) float x[kDim];   // x, then the normalized input
    alignas(16) float g[kDim];
    uint64_t full[kRing];
    uint64_t empty[kRing];
    unsigned long long best[kConsumerWarps];
    float scale;
    int last;
};
static_assert(sizeof(HeadSmem) + 1024 <= 232448, "shared memory per CTA");

__device__ __forceinline__ uint32_t su32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false after about 2 s (the caller records a status bit).
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity) {
    if (bar_try(b, parity)) {
        return true;
    }
    unsigned long long t0;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t0));
    while (true) {
        for (int i = 0; i < 64; ++i) {
            if (bar_try(b, parity)) {
                return true;
            }
        }
        unsigned long long t;
        asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
        if (t - t0 > kHeadWaitNs) {
            return false;
        }
    }
}

__global__ void head_pack_kernel(const uint8_t *__restrict__ gguf, uint8_t *__restrict__ packed,
                                 uint8_t *__restrict__ rowflag, size_t rows) {
    const size_t blocks = rows * kQ8Blocks;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < blocks; i += size_t(gridDim.x) * blockDim.x) {
        const size_t r = i / kQ8Blocks;
        const int b = int(i - r * kQ8Blocks);
        const uint8_t *src = gguf + r * kQ8RowBytes + size_t(b) * 34;
        uint8_t *row = packed + r * kPackedRowBytes;
        row[kDim + 2 * b] = src[0];
        row[kDim + 2 * b + 1] = src[1];
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            row[32 * b + j] = src[2 + j];
        }
        if (b == 0) {
            for (int j = kDim + 2 * kQ8Blocks; j < kPackedRowBytes; ++j) {
                row[j] = 0;
            }
        }
        // rows holding an infinite scale take the plain product path
        if ((src[1] & 0x7Cu) == 0x7Cu && (src[1] & 0x03u) == 0u && src[0] == 0u) {
            rowflag[r] = 1u;
        }
    }
}

__global__ void head_unpack_kernel(const uint8_t *__restrict__ packed, uint8_t *__restrict__ gguf, size_t rows) {
    const size_t blocks = rows * kQ8Blocks;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < blocks; i += size_t(gridDim.x) * blockDim.x) {
        const size_t r = i / kQ8Blocks;
        const int b = int(i - r * kQ8Blocks);
        uint8_t *dst = gguf + r * kQ8RowBytes + size_t(b) * 34;
        const uint8_t *row = packed + r * kPackedRowBytes;
        dst[0] = row[kDim + 2 * b];
        dst[1] = row[kDim + 2 * b + 1];
        for (int j = 0; j < 32; ++j) {
            dst[2 + j] = row[32 * b + j];
        }
    }
}

// Order key of a logit for the greedy argmax: larger values first, then the
// lower row (-0 and +0 compare equal, as the reference's ">" does).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t row) {
    uint32_t b = __float_as_uint(v + 0.0f);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - row);
}

// One row's four chains of this lane (elements 4 sub .. 4 sub + 3 of every
// block) from a staged packed row.
__device__ __forceinline__ void row_chains(const uint8_t *row, const float *xn, int sub, bool plain, float (&acc)[4]) {
    const uint32_t *q32 = reinterpret_cast<const uint32_t *>(row);
    const unsigned short *sc = reinterpret_cast<const unsigned short *>(row + kDim);
    if (!plain) {
#pragma unroll 6
        for (int b = 0; b < kQ8Blocks; ++b) {
            const uint32_t u = q32[8 * b + sub] ^ 0x80808080u;  // q + 128 per byte
            const float s = __half2float(__ushort_as_half(sc[b]));
            const float s1 = __fmul_rn(s, 0.00390625f);  // s / 256, exact
            const float s2 = __fmul_rn(s, -32896.0f);    // -(2^15 + 128) s, exact
            const float4 xv = *reinterpret_cast<const float4 *>(xn + 32 * b + 4 * sub);
            const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                // 2^23 + 256 u: byte 1 = u, byte 3 = 0x4B
                const uint32_t m = __byte_perm(u, 0x4B000000u, 0x7504u | (uint32_t(k) << 4));
                const float w = __fmaf_rn(__uint_as_float(m), s1, s2);  // q * s, exact
                acc[k] = __fadd_rn(acc[k], __fmul_rn(w, xs[k]));
            }
        }
    } else {
        // a row with an infinite scale: the products themselves (0 * inf is
        // NaN, as in the reference; the FMA form would give NaN for every q)
        for (int b = 0; b < kQ8Blocks; ++b) {
            const uint32_t q = q32[8 * b + sub];
            const float s = __half2float(__ushort_as_half(sc[b]));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float w = __fmul_rn(float(int(int8_t((q >> (8 * k)) & 0xFFu))), s);
                acc[k] = __fadd_rn(acc[k], __fmul_rn(w, xn[32 * b + 4 * sub + k]));
            }
        }
    }
}

// The head in one persistent launch (one CTA per SM): every CTA normalizes
// x itself (the 2880-term chain runs on one thread while the producer warp
// streams the CTA's first row stages in), then its consumer warps compute
// the rows of stages blockIdx.x, blockIdx.x + grid, ... from the ring.
__global__ void __launch_bounds__(kHeadThreads, 1)
    head_kernel(const uint8_t *__restrict__ w, const uint8_t *__restrict__ rowflag, uint32_t rows,
                const float *__restrict__ x, const float *__restrict__ g, HeadState *st, float *__restrict__ logits,
                int32_t *__restrict__ token_out) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    HeadSmem &s = *reinterpret_cast<HeadSmem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t stages = (rows + kStageRows - 1) / kStageRows;
    const uint32_t mine = (stages > blockIdx.x) ? (stages - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRing; ++i) {
            bar_init(&s.full[i], 1);
            bar_init(&s.empty[i], 2);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == kProducerWarp) {
        if (lane == 0) {
            // the matrix is read once per call: its lines go first from L2
            uint64_t pol;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
            for (uint32_t j = 0; j < mine; ++j) {
                const uint32_t slot = j % kRing;
                if (j >= kRing && !bar_wait(&s.empty[slot], ((j / kRing) - 1) & 1)) {
                    atomicOr(&st->status, 1u);
                    break;
                }
                const uint32_t stage = blockIdx.x + j * gridDim.x;
                const uint32_t r0 = stage * kStageRows;
                const uint32_t n = min(rows, r0 + kStageRows) - r0;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&s.full[slot])),
                             "r"(n * kPackedRowBytes)
                             : "memory");
                for (uint32_t k = 0; k < n; ++k) {
                    asm volatile(
                        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
                        "%2, [%3], %4;" ::"r"(su32(&s.ring[slot][k * kSmemRowStride])),
                        "l"(w + size_t(r0 + k) * kPackedRowBytes), "r"(uint32_t(kPackedRowBytes)),
                        "r"(su32(&s.full[slot])), "l"(pol)
                        : "memory");
                }
            }
            // every copy this CTA issued lands before it exits
            for (uint32_t k = 0; k < kRing && k < mine; ++k) {
                const uint32_t j = mine - 1 - k;
                bar_wait(&s.full[j % kRing], (j / kRing) & 1);
            }
        }
        return;
    }
    // ---- consumer warps: normalize, then rows ----
    for (int k = threadIdx.x; k < kDim; k += 32 * kConsumerWarps) {
        s.x[k] = x[k];
        s.g[k] = g[k];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumerWarps) : "memory");
    if (threadIdx.x == 0) {
        // rms_norm (src/tensor.cpp:568-580): the sum of squares in order
        float sum = 0.0f;
#pragma unroll 16
        for (int k = 0; k < kDim; ++k) {
            sum = __fadd_rn(sum, __fmul_rn(s.x[k], s.x[k]));
        }
        s.scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, float(kDim)), 1.0e-5f)));
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumerWarps) : "memory");
    const float scale = s.scale;
    for (int k = threadIdx.x; k < kDim; k += 32 * kConsumerWarps) {
        s.x[k] = __fmul_rn(__fmul_rn(s.x[k], scale), s.g[k]);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumerWarps) : "memory");

    const int slot = warp >> 1;        // this warp's ring slot
    const int half = warp & 1;         // rows 4 half .. 4 half + 3 of the stage
    const int sub = lane & 7;          // elements 4 sub .. 4 sub + 3 of every block
    unsigned long long best = 0ull;
    for (uint32_t j = uint32_t(slot); j < mine; j += kRing) {
        if (!bar_wait(&s.full[slot], (j / kRing) & 1)) {
            atomicOr(&st->status, 1u);
            break;
        }
        const uint32_t stage = blockIdx.x + j * gridDim.x;
        const uint32_t r = stage * kStageRows + 4 * half + uint32_t(lane >> 3);
        const bool live = r < rows;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint8_t *row = &s.ring[slot][(4 * half + (lane >> 3)) * kSmemRowStride];
        row_chains(row, s.x, sub, live && rowflag[r], acc);
        __syncwarp();
        if (lane == 0) {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&s.empty[slot])) : "memory");
        }
        // acc[j] = chain j + chain j + 16 (sub 0..3 take sub 4..7's), then the
        // 16 values in order from 0.0f, handed from sub 0 to sub 3
        float a[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a[k] = __fadd_rn(acc[k], __shfl_down_sync(0xffffffffu, acc[k], 4));
        }
        float total = 0.0f;
#pragma unroll
        for (int hop = 0; hop < 4; ++hop) {
            if (sub == hop) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    total = __fadd_rn(total, a[k]);
                }
            }
            if (hop < 3) {
                total = __shfl_up_sync(0xffffffffu, total, 1);
            }
        }
        if (sub == 3 && live) {
            if (logits) {
                logits[r] = total;
            }
            if (total == total) {
                const unsigned long long k = argmax_key(total, r);
                best = (k > best) ? k : best;
            } else if (r == 0) {
                atomicExch(&st->nan0, 1u);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
        best = (o > best) ? o : best;
    }
    if (lane == 0) {
        s.best[warp] = best;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumerWarps) : "memory");
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int k = 0; k < kConsumerWarps; ++k) {
            b = (s.best[k] > b) ? s.best[k] : b;
        }
        if (b) {
            atomicMax(&st->key, b);
        }
        __threadfence();
        s.last = (atomicAdd(&st->arrived, 1u) == gridDim.x - 1) ? 1 : 0;
        if (s.last) {
            __threadfence();
            const unsigned long long k = atomicAdd(&st->key, 0ull);
            const unsigned int nan0 = atomicAdd(&st->nan0, 0u);
            // greedy starts at row 0: a NaN there is never replaced, and with
            // no number at all row 0 stays too
            const int32_t tok = (!nan0 && k != 0ull) ? int32_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull)) : 0;
            st->token = tok;
            if (token_out) {
                *token_out = tok;
            }
            st->key = 0ull;
            st->nan0 = 0u;
            __threadfence();
            st->arrived = 0u;
        }
    }
}

int grid_for_head(size_t n) {
    return int((n + 255) / 256 > 148 * 16 ? 148 * 16 : (n + 255) / 256);
}

} // namespace
} // namespace ttl

using namespace ttl;

struct ttl_head {
    int device = 0;
    uint32_t vocab = 0;
    cudaStream_t stream = nullptr;
    uint8_t *w = nullptr;      // packed rows [vocab][3072]
    uint8_t *rowflag = nullptr;  // [vocab] 1: the row holds an infinite scale
    int sms = 148;
    float *g = nullptr;        // output_norm.weight [2880]
    HeadState *st = nullptr;
    float *d_x = nullptr;      // host-call staging
    float *d_logits = nullptr;
    float *pin = nullptr;      // pinned host staging: x [2880], then token
    bool uploaded = false;
    std::string error;
};

namespace {

int head_fail(ttl_head *h, int code, const std::string &msg) {
    if (h) {
        h->error = msg;
    }
    return ttl::fail(nullptr, code, msg);
}

#define TTL_HEAD_CUDA(h, expr)                                                                          \
    do {                                                                                                \
        const cudaError_t e_ = (expr);                                                                  \
        if (e_ != cudaSuccess) {                                                                        \
            return head_fail((h), TTL_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));    \
        }                                                                                               \
    } while (0)

int head_enqueue(ttl_head *h, const float *x, float *logits, int32_t *token) {
    const size_t smem = sizeof(HeadSmem) + 1024;
    head_kernel<<<h->sms, kHeadThreads, smem, h->stream>>>(h->w, h->rowflag, h->vocab, x, h->g, h->st, logits, token);
    TTL_HEAD_CUDA(h, cudaGetLastError());
    return TTL_OK;
}

// The status word a kernel sets when a bounded wait gives up: read, cleared
// and reported (the call's results are not valid then).
int check_head_status(ttl_head *h) {
    uint32_t status = 0;
    TTL_HEAD_CUDA(h, cudaMemcpy(&status, &h->st->status, sizeof(status), cudaMemcpyDeviceToHost));
    if (status) {
        cudaMemset(&h->st->status, 0, sizeof(uint32_t));
        return head_fail(h, TTL_ERR_DEVICE, "output head: a bounded wait gave up");
    }
    return TTL_OK;
}

} // namespace

extern "C" {

int ttl_head_create(int device, uint32_t vocab, ttl_head **out) {
    if (!out) {
        return head_fail(nullptr, TTL_ERR_ARGUMENT, "null handle pointer");
    }
    *out = nullptr;
    if (vocab == 0 || vocab > (1u << 24)) {
        return head_fail(nullptr, TTL_ERR_ARGUMENT, "vocab must be in 1..2^24");
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return head_fail(nullptr, TTL_ERR_UNSUPPORTED, "no CUDA device");
    }
    if (device < 0 && cudaGetDevice(&device) != cudaSuccess) {
        return head_fail(nullptr, TTL_ERR_CUDA, "cudaGetDevice failed");
    }
    if (device >= count) {
        return head_fail(nullptr, TTL_ERR_ARGUMENT, "device ordinal out of range");
    }
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
        return head_fail(nullptr, TTL_ERR_UNSUPPORTED, "the kernels are built for sm_100a (B200)");
    }
    ttl_head *h = new ttl_head();
    h->device = device;
    h->vocab = vocab;
    h->sms = prop.multiProcessorCount;
    auto bail = [&](int rc) {
        ttl_head_destroy(h);
        return rc;
    };
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&h->w, size_t(vocab) * kPackedRowBytes) != cudaSuccess ||
        cudaMalloc(&h->rowflag, vocab) != cudaSuccess ||
        cudaMalloc(&h->g, kDim * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->st, sizeof(HeadState)) != cudaSuccess ||
        cudaMalloc(&h->d_x, kDim * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->d_logits, size_t(vocab) * sizeof(float)) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void **>(&h->pin), (kDim + 4) * sizeof(float), cudaHostAllocDefault) !=
            cudaSuccess ||
        cudaMemset(h->st, 0, sizeof(HeadState)) != cudaSuccess ||
        cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(sizeof(HeadSmem) + 1024)) != cudaSuccess) {
        cudaGetLastError();
        return bail(head_fail(nullptr, TTL_ERR_CUDA, "output head: device allocation failed"));
    }
    *out = h;
    return TTL_OK;
}

void ttl_head_destroy(ttl_head *h) {
    if (!h) {
        return;
    }
    cudaSetDevice(h->device);
    if (h->stream) {
        cudaStreamSynchronize(h->stream);
        cudaStreamDestroy(h->stream);
    }
    cudaFree(h->w);
    cudaFree(h->rowflag);
    cudaFree(h->g);
    cudaFree(h->st);
    cudaFree(h->d_x);
    cudaFree(h->d_logits);
    if (h->pin) {
        cudaFreeHost(h->pin);
    }
    delete h;
}

const char *ttl_head_last_error(const ttl_head *h) {
    return h ? h->error.c_str() : ttl::thread_error().c_str();
}

int ttl_head_upload(ttl_head *h, const void *q8_0, const float *norm_w) {
    if (!h || !q8_0 || !norm_w) {
        return head_fail(h, TTL_ERR_ARGUMENT, "null argument");
    }
    TTL_HEAD_CUDA(h, cudaSetDevice(h->device));
    const size_t gguf_bytes = size_t(h->vocab) * kQ8RowBytes;
    const uint8_t *src = static_cast<const uint8_t *>(q8_0);
    uint8_t *staging = nullptr;
    if (!is_device_pointer(q8_0)) {
        TTL_HEAD_CUDA(h, cudaMalloc(&staging, gguf_bytes));
        const cudaError_t e = cudaMemcpy(staging, q8_0, gguf_bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(staging);
            return head_fail(h, TTL_ERR_CUDA, std::string("weight copy: ") + cudaGetErrorString(e));
        }
        src = staging;
    }
    cudaError_t e0 = cudaMemsetAsync(h->rowflag, 0, h->vocab, h->stream);
    head_pack_kernel<<<grid_for_head(size_t(h->vocab) * kQ8Blocks), 256, 0, h->stream>>>(src, h->w, h->rowflag,
                                                                                          h->vocab);
    const cudaError_t e1 = (e0 != cudaSuccess) ? e0 : cudaGetLastError();
    const cudaError_t e2 = cudaMemcpyAsync(h->g, norm_w, kDim * sizeof(float), cudaMemcpyDefault, h->stream);
    const cudaError_t e3 = cudaStreamSynchronize(h->stream);
    if (staging) {
        cudaFree(staging);
    }
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess) {
        return head_fail(h, TTL_ERR_CUDA, "output head upload failed");
    }
    h->uploaded = true;
    return TTL_OK;
}

int ttl_head_unpack(ttl_head *h, void *gguf_out) {
    if (!h || !gguf_out) {
        return head_fail(h, TTL_ERR_ARGUMENT, "null argument");
    }
    if (!h->uploaded) {
        return head_fail(h, TTL_ERR_STATE, "output head not uploaded");
    }
    TTL_HEAD_CUDA(h, cudaSetDevice(h->device));
    const size_t gguf_bytes = size_t(h->vocab) * kQ8RowBytes;
    uint8_t *dst = static_cast<uint8_t *>(gguf_out);
    uint8_t *staging = nullptr;
    if (!is_device_pointer(gguf_out)) {
        TTL_HEAD_CUDA(h, cudaMalloc(&staging, gguf_bytes));
        dst = staging;
    }
    head_unpack_kernel<<<grid_for_head(size_t(h->vocab) * kQ8Blocks), 256, 0, h->stream>>>(h->w, dst, h->vocab);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
        e = cudaStreamSynchronize(h->stream);
    }
    if (e == cudaSuccess && staging) {
        e = cudaMemcpy(gguf_out, staging, gguf_bytes, cudaMemcpyDeviceToHost);
    }
    if (staging) {
        cudaFree(staging);
    }
    if (e != cudaSuccess) {
        return head_fail(h, TTL_ERR_CUDA, std::string("output head unpack: ") + cudaGetErrorString(e));
    }
    return TTL_OK;
}

int ttl_head_forward_async(ttl_head *h, const float *x, float *logits, int32_t *token) {
    if (!h || !x) {
        return head_fail(h, TTL_ERR_ARGUMENT, "null argument");
    }
    if (!h->uploaded) {
        return head_fail(h, TTL_ERR_STATE, "output head not uploaded");
    }
    TTL_HEAD_CUDA(h, cudaSetDevice(h->device));
    return head_enqueue(h, x, logits, token);
}

int ttl_head_forward(ttl_head *h, const float *x, float *logits, int32_t *token) {
    if (!h || !x || (!logits && !token)) {
        return head_fail(h, TTL_ERR_ARGUMENT, "null argument");
    }
    if (!h->uploaded) {
        return head_fail(h, TTL_ERR_STATE, "output head not uploaded");
    }
    TTL_HEAD_CUDA(h, cudaSetDevice(h->device));
    std::memcpy(h->pin, x, kDim * sizeof(float));
    TTL_HEAD_CUDA(h, cudaMemcpyAsync(h->d_x, h->pin, kDim * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    int32_t *tok_dev = &h->st->token;
    const int rc = head_enqueue(h, h->d_x, logits ? h->d_logits : nullptr, nullptr);
    if (rc) {
        return rc;
    }
    int32_t *tok_pin = reinterpret_cast<int32_t *>(h->pin + kDim);
    TTL_HEAD_CUDA(h, cudaMemcpyAsync(tok_pin, tok_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, h->stream));
    if (logits) {
        TTL_HEAD_CUDA(h, cudaMemcpyAsync(logits, h->d_logits, size_t(h->vocab) * sizeof(float), cudaMemcpyDeviceToHost,
                                         h->stream));
    }
    TTL_HEAD_CUDA(h, cudaStreamSynchronize(h->stream));
    if (token) {
        *token = *tok_pin;
    }
    return check_head_status(h);
}

int ttl_head_sync(ttl_head *h) {
    if (!h) {
        return head_fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    TTL_HEAD_CUDA(h, cudaSetDevice(h->device));
    TTL_HEAD_CUDA(h, cudaStreamSynchronize(h->stream));
    return check_head_status(h);
}

void *ttl_head_stream(ttl_head *h) {
    return h ? static_cast<void *>(h->stream) : nullptr;
}

} // extern "C"
