// decode.cu -- decode (T = 1) MoE kernels: router + top-4 + softmax, fused
// gate/up matvec + SwiGLU, down matvec + weighted combine (+ residual).
//
// Reference: GptOssModel::moe, tt-lab src/model.cpp:292-338, with the kernels
// matvec_add_f32 (src/tensor.cpp:186-200) and matvec_add_mxfp4_2880
// (src/tensor.cpp:239-304).
//
// Expert matvecs are warp-cooperative fused dequant-GEMVs: one warp per output
// row, lanes split the 90 K-blocks (lane l takes blocks l, l+32, l+64), every
// lane streams 16-byte vectors of packed E2M1 nibbles, converts pairs with the
// sm_100 cvt.rn.f16x2.e2m1x2 instruction, accumulates the 32-element block in
// f32 and applies the block's E8M0 scale once; a butterfly reduction finishes
// the row.  Gate and up rows of the same index are done by the same warp so the
// SwiGLU is applied in registers.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ttl {
namespace {

constexpr int kRouterThreads = 192;  // 15 contiguous columns per thread
constexpr int kRouterChunk = kDim / kRouterThreads;
constexpr int kXStride = 36;         // padded floats per K-block in shared memory
constexpr int kMatvecThreads = 512;
constexpr int kDownThreads = 512;

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_u8(const uint8_t *p) {
    return __ldg(p);
}

template <int N> __device__ __forceinline__ double block_sum_d(double v, double *scratch) {
    v = warp_sum_d(v);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) {
        scratch[warp] = v;
    }
    __syncthreads();
    double total = 0.0;
#pragma unroll
    for (int i = 0; i < N / 32; ++i) {
        total += scratch[i];
    }
    return total;
}

// Exclusive prefix sum across the block (f64), deterministic order.
template <int N> __device__ __forceinline__ double block_exclusive_scan_d(double v, double *scratch) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    double inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) {
            inc += t;
        }
    }
    __syncthreads();
    if (lane == 31) {
        scratch[warp] = inc;
    }
    __syncthreads();
    double base = 0.0;
    for (int i = 0; i < warp; ++i) {
        base += scratch[i];
    }
    return base + inc - v;
}

// Dot of one 32-element block (16 packed bytes in `q`) with xs[0..31].
__device__ __forceinline__ float block_dot(const uint4 q, const float *xb) {
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    float acc0 = 0.0f;
    float acc1 = 0.0f;
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
        const float4 xa = *reinterpret_cast<const float4 *>(xb + wd * 8);
        const float4 xc = *reinterpret_cast<const float4 *>(xb + wd * 8 + 4);
        const float2 v0 = __half22float2(e2m1x2_to_half2(words[wd] & 0xffu));
        const float2 v1 = __half22float2(e2m1x2_to_half2((words[wd] >> 8) & 0xffu));
        const float2 v2 = __half22float2(e2m1x2_to_half2((words[wd] >> 16) & 0xffu));
        const float2 v3 = __half22float2(e2m1x2_to_half2(words[wd] >> 24));
        acc0 = fmaf(v0.x, xa.x, acc0);
        acc1 = fmaf(v0.y, xa.y, acc1);
        acc0 = fmaf(v1.x, xa.z, acc0);
        acc1 = fmaf(v1.y, xa.w, acc1);
        acc0 = fmaf(v2.x, xc.x, acc0);
        acc1 = fmaf(v2.y, xc.y, acc1);
        acc0 = fmaf(v3.x, xc.z, acc0);
        acc1 = fmaf(v3.y, xc.w, acc1);
    }
    return acc0 + acc1;
}

// Reference selection sort (src/model.cpp:296-309) on `vals`.
__device__ void select_top4_ref(const float *vals, int experts, int32_t idx[4]) {
    uint8_t order[kMaxExperts];
    for (int i = 0; i < experts; ++i) {
        order[i] = uint8_t(i);
    }
    for (int i = 0; i < kTopK; ++i) {
        int best = i;
        for (int j = i + 1; j < experts; ++j) {
            if (vals[order[j]] > vals[order[best]]) {
                best = j;
            }
        }
        const uint8_t t = order[i];
        order[i] = order[best];
        order[best] = t;
        idx[i] = order[i];
    }
}

// Softmax over the 4 selected logits (src/model.cpp:310-321).
__device__ void softmax4_ref(const float sel[4], float out[4]) {
    float maximum = -INFINITY;
    for (int i = 0; i < kTopK; ++i) {
        maximum = (maximum < sel[i]) ? sel[i] : maximum;
    }
    float sum = 0.0f;
    for (int i = 0; i < kTopK; ++i) {
        out[i] = expf(__fsub_rn(sel[i], maximum));
        sum = __fadd_rn(sum, out[i]);
    }
    for (int i = 0; i < kTopK; ++i) {
        out[i] = __fdiv_rn(out[i], sum);
    }
}

// The reference router logit of expert e exactly: bias first, then products
// rounded to f32 and added in column order (src/tensor.cpp:193-198).
__device__ float exact_logit(const float *__restrict__ wrow, float bias, const float *hs) {
    float s = bias;
    for (int c = 0; c < kDim; c += 8) {
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            p[j] = __fmul_rn(__ldg(wrow + c + j), hs[c + j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s = __fadd_rn(s, p[j]);
        }
    }
    return s;
}

// One CTA per expert computes its logit with an f64 sum of the f32-rounded
// products and a bound on how far the reference's sequential f32 chain can be
// from it: |R - T| <= u * sum_c |s_c| (s_c the chain's partial sums, u = 2^-24),
// with s_c taken from the exact prefix sums.  The last CTA to finish selects
// the top 4.  If any selected expert's interval overlaps another expert's, the
// experts that could reach the top 4 are re-evaluated exactly in the
// reference's order and the reference's selection sort decides, so the indices
// equal the reference's bit for bit.
__global__ void __launch_bounds__(kRouterThreads) decode_router_kernel(LayerDev L, DecodeWork w, int experts,
                                                                       const float *__restrict__ x, int mode) {
    __shared__ float hs[kDim];
    __shared__ double scratch[kRouterThreads / 32];
    __shared__ float s_logit[kMaxExperts];
    __shared__ float s_bound[kMaxExperts];
    __shared__ float s_val[kMaxExperts];
    __shared__ int s_last;
    __shared__ int s_amb;
    __shared__ int32_t s_idx[4];

    const int e = blockIdx.x;
    const int t = threadIdx.x;
    const int c0 = t * kRouterChunk;

    if (mode == 0) {
#pragma unroll
        for (int j = 0; j < kRouterChunk; ++j) {
            hs[c0 + j] = x[c0 + j];
        }
    } else {
        // RMSNorm (src/tensor.cpp:568-580): scale = 1 / sqrt(sum(x^2) / n + eps),
        // out = (x * scale) * weight.  The sum of squares is formed in f64.
        double ss = 0.0;
        float xv[kRouterChunk];
#pragma unroll
        for (int j = 0; j < kRouterChunk; ++j) {
            xv[j] = x[c0 + j];
            ss += double(__fmul_rn(xv[j], xv[j]));
        }
        const float sum = float(block_sum_d<kRouterThreads>(ss, scratch));
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, float(kDim)), 1.0e-5f)));
#pragma unroll
        for (int j = 0; j < kRouterChunk; ++j) {
            hs[c0 + j] = __fmul_rn(__fmul_rn(xv[j], scale), L.norm_w[c0 + j]);
        }
    }
    __syncthreads();
    if (e == 0) {
#pragma unroll
        for (int j = 0; j < kRouterChunk; ++j) {
            w.h[c0 + j] = hs[c0 + j];
        }
    }

    const float *wr = L.router_w + size_t(e) * kDim;
    const float bias = L.router_b[e];
    float p[kRouterChunk];
    double local = 0.0;
#pragma unroll
    for (int j = 0; j < kRouterChunk; ++j) {
        p[j] = __fmul_rn(__ldg(wr + c0 + j), hs[c0 + j]);
        local += double(p[j]);
    }
    const double before = block_exclusive_scan_d<kRouterThreads>(local, scratch);
    double run = double(bias) + before;
    double abs_sum = 0.0;
#pragma unroll
    for (int j = 0; j < kRouterChunk; ++j) {
        run += double(p[j]);
        abs_sum += fabs(run);
    }
    const double total = block_sum_d<kRouterThreads>(local, scratch);
    const double abs_total = block_sum_d<kRouterThreads>(abs_sum, scratch);
    if (t == 0) {
        const double logit = double(bias) + total;
        const float lf = float(logit);
        // 1.02 * u * sum|s_c| + u * |T| (rounding of T to f32) + tiny.
        const double bound = 1.02 * 5.9604644775390625e-08 * abs_total + 5.9604644775390625e-08 * fabs(logit) + 1e-30;
        w.logits[e] = lf;
        w.bounds[e] = float(bound * 1.0001);
        __threadfence();
        const unsigned int arrived = atomicAdd(w.arrive, 1u);
        s_last = (arrived == unsigned(experts - 1));
    }
    __syncthreads();
    if (!s_last) {
        return;
    }
    __threadfence();
    for (int i = t; i < experts; i += kRouterThreads) {
        s_logit[i] = __ldcg(w.logits + i);
        s_bound[i] = __ldcg(w.bounds + i);
        s_val[i] = s_logit[i];
    }
    if (t == 0) {
        *w.arrive = 0u;  // ready for the next launch
        s_amb = 0;
    }
    __syncthreads();

    // Fast top 4 by value (warp 0); ties only matter when flagged below.
    if (t < 32) {
        int chosen[4];
        for (int r = 0; r < kTopK; ++r) {
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int i = t; i < experts; i += 32) {
                bool taken = false;
                for (int q = 0; q < r; ++q) {
                    taken |= (chosen[q] == i);
                }
                const float v = s_logit[i];
                if (!taken && (v > bv || (v == bv && i < bi) || bi == 0x7fffffff)) {
                    bv = v;
                    bi = i;
                }
            }
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi == 0x7fffffff) {
                bi = r;  // all candidates NaN: let the exact path decide
                chosen[r] = bi;
                s_amb = 1;
            }
            chosen[r] = bi;
        }
        // Ambiguity: any selected a and other b whose intervals touch.
        bool amb = false;
        for (int i = t; i < experts; i += 32) {
            for (int q = 0; q < kTopK; ++q) {
                const int a = chosen[q];
                if (a != i && !(s_logit[a] != s_logit[a])) {
                    const float gap = fabsf(s_logit[a] - s_logit[i]);
                    if (!(gap > s_bound[a] + s_bound[i])) {
                        amb = true;
                    }
                }
            }
        }
        amb = __any_sync(0xffffffffu, amb);
        if (t == 0) {
            s_amb = (amb || s_amb) ? 1 : 0;
            for (int q = 0; q < kTopK; ++q) {
                s_idx[q] = chosen[q];
            }
        }
    }
    __syncthreads();

    if (s_amb) {
        // Lower edge of the selected intervals; experts whose upper edge
        // reaches it are re-evaluated exactly.
        float lower = INFINITY;
        for (int q = 0; q < kTopK; ++q) {
            lower = fminf(lower, s_logit[s_idx[q]] - s_bound[s_idx[q]]);
        }
        for (int i = t; i < experts; i += kRouterThreads) {
            if (!(s_logit[i] + s_bound[i] < lower)) {
                s_val[i] = exact_logit(L.router_w + size_t(i) * kDim, L.router_b[i], hs);
            }
        }
        __syncthreads();
        if (t == 0) {
            int32_t idx[4];
            select_top4_ref(s_val, experts, idx);
            for (int q = 0; q < kTopK; ++q) {
                s_idx[q] = idx[q];
            }
            atomicAdd(&w.counters[0], 1ull);
        }
        __syncthreads();
    }
    if (t == 0) {
        float sel[4], wt[4];
        for (int q = 0; q < kTopK; ++q) {
            sel[q] = s_val[s_idx[q]];
        }
        softmax4_ref(sel, wt);
        for (int q = 0; q < kTopK; ++q) {
            w.top_idx[q] = s_idx[q];
            w.top_w[q] = wt[q];
        }
    }
}

// Loads a 2880-float vector into the padded shared layout [90][36].
__device__ __forceinline__ void load_padded(float *xs, const float *__restrict__ v) {
    for (int i = threadIdx.x; i < kDim / 4; i += blockDim.x) {
        const float4 q = *reinterpret_cast<const float4 *>(v + 4 * i);
        const int kb = (4 * i) >> 5;
        const int off = (4 * i) & 31;
        *reinterpret_cast<float4 *>(xs + kb * kXStride + off) = q;
    }
}

__global__ void __launch_bounds__(kMatvecThreads, 1) decode_gateup_kernel(LayerDev L, DecodeWork w, DecodeShape s) {
    __shared__ __align__(16) float xs[kBlocks * kXStride];
    __shared__ int local[4];
    load_padded(xs, w.h);
    if (threadIdx.x < kTopK) {
        const int e = w.top_idx[threadIdx.x];
        int le = e - s.expert_begin;
        if (e < 0 || e >= s.experts) {
            set_status(w.status, kStatusBadExpert);
            le = -1;
        }
        local[threadIdx.x] = (le >= 0 && le < s.expert_count) ? le : -1;
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kMatvecThreads / 32);
    for (int item = blockIdx.x * (kMatvecThreads / 32) + (threadIdx.x >> 5); item < kTopK * kDim; item += warps) {
        const int sel = item / kDim;
        const int row = item - sel * kDim;
        const int le = local[sel];
        if (le < 0) {
            continue;
        }
        const uint8_t *gm = L.gate + size_t(le) * kPackedMatrixBytes;
        const uint8_t *um = L.up + size_t(le) * kPackedMatrixBytes;
        uint4 gq[3], uq[3];
        uint32_t gsb[3], usb[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int kb = lane + 32 * j;
            if (kb < kBlocks) {
                gq[j] = ldg_stream(gm + size_t(row) * kNibbleRowBytes + kb * 16);
                uq[j] = ldg_stream(um + size_t(row) * kNibbleRowBytes + kb * 16);
                gsb[j] = ldg_u8(gm + scale_offset(row, kb));
                usb[j] = ldg_u8(um + scale_offset(row, kb));
            }
        }
        float ag = 0.0f;
        float au = 0.0f;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int kb = lane + 32 * j;
            if (kb < kBlocks) {
                const float *xb = xs + kb * kXStride;
                ag = fmaf(e8m0_ref_scale(gsb[j]), 2.0f * block_dot(gq[j], xb), ag);
                au = fmaf(e8m0_ref_scale(usb[j]), 2.0f * block_dot(uq[j], xb), au);
            }
        }
        ag = warp_sum(ag);
        au = warp_sum(au);
        if (lane == 0) {
            const float g = __fadd_rn(L.gate_b[size_t(le) * kDim + row], ag);
            const float u = __fadd_rn(L.up_b[size_t(le) * kDim + row], au);
            w.hidden[size_t(sel) * kDim + row] = swiglu_ref(g, u);
        }
    }
}

__global__ void __launch_bounds__(kDownThreads, 1)
    decode_down_kernel(LayerDev L, DecodeWork w, DecodeShape s, const float *__restrict__ residual,
                       float *__restrict__ out) {
    extern __shared__ __align__(16) float hsm[];  // [4][90][36]
    __shared__ int local[4];
    __shared__ float wts[4];
    for (int sel = 0; sel < kTopK; ++sel) {
        load_padded(hsm + sel * kBlocks * kXStride, w.hidden + size_t(sel) * kDim);
    }
    if (threadIdx.x < kTopK) {
        const int e = w.top_idx[threadIdx.x];
        const int le = e - s.expert_begin;
        local[threadIdx.x] = (e >= 0 && e < s.experts && le >= 0 && le < s.expert_count) ? le : -1;
        wts[threadIdx.x] = w.top_w[threadIdx.x];
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kDownThreads / 32);
    for (int row = blockIdx.x * (kDownThreads / 32) + (threadIdx.x >> 5); row < kDim; row += warps) {
        uint4 q[4][3];
        uint32_t sb[4][3];
#pragma unroll
        for (int sel = 0; sel < kTopK; ++sel) {
            const int le = local[sel];
            const uint8_t *m = L.down + size_t(le < 0 ? 0 : le) * kPackedMatrixBytes;
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int kb = lane + 32 * j;
                if (le >= 0 && kb < kBlocks) {
                    q[sel][j] = ldg_stream(m + size_t(row) * kNibbleRowBytes + kb * 16);
                    sb[sel][j] = ldg_u8(m + scale_offset(row, kb));
                }
            }
        }
        float acc[4];
#pragma unroll
        for (int sel = 0; sel < kTopK; ++sel) {
            float a = 0.0f;
            if (local[sel] >= 0) {
#pragma unroll
                for (int j = 0; j < 3; ++j) {
                    const int kb = lane + 32 * j;
                    if (kb < kBlocks) {
                        a = fmaf(e8m0_ref_scale(sb[sel][j]),
                                 2.0f * block_dot(q[sel][j], hsm + sel * kBlocks * kXStride + kb * kXStride), a);
                    }
                }
            }
            acc[sel] = warp_sum(a);
        }
        if (lane == 0) {
            // Combine in rank order: out += w * (bias + dot), product rounded
            // first (src/model.cpp:323, :333-336).
            float o = 0.0f;
#pragma unroll
            for (int sel = 0; sel < kTopK; ++sel) {
                const int le = local[sel];
                if (le >= 0) {
                    const float d = __fadd_rn(L.down_b[size_t(le) * kDim + row], acc[sel]);
                    o = __fadd_rn(o, __fmul_rn(wts[sel], d));
                }
            }
            out[row] = residual ? __fadd_rn(residual[row], o) : o;
        }
    }
}

__global__ void add_kernel(const float *a, const float *b, float *out, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        out[i] = __fadd_rn(a[i], b[i]);
    }
}

} // namespace

void launch_decode_router(const LayerDev &L, const DecodeWork &w, const DecodeShape &s, const float *x, int mode,
                          cudaStream_t stream) {
    decode_router_kernel<<<s.experts, kRouterThreads, 0, stream>>>(L, w, s.experts, x, mode);
}

void launch_decode_gateup(const LayerDev &L, const DecodeWork &w, const DecodeShape &s, cudaStream_t stream) {
    decode_gateup_kernel<<<s.sms, kMatvecThreads, 0, stream>>>(L, w, s);
}

void configure_decode_kernels() {
    const int smem = kTopK * kBlocks * kXStride * int(sizeof(float));
    cudaFuncSetAttribute(decode_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

void launch_decode_down(const LayerDev &L, const DecodeWork &w, const DecodeShape &s, const float *residual,
                        float *out, cudaStream_t stream) {
    const int smem = kTopK * kBlocks * kXStride * int(sizeof(float));
    const int grid = (kDim + kDownThreads / 32 - 1) / (kDownThreads / 32);
    decode_down_kernel<<<grid, kDownThreads, smem, stream>>>(L, w, s, residual, out);
}

void launch_add(const float *residual, const float *moe, float *out, int n, cudaStream_t stream) {
    add_kernel<<<(n + 255) / 256, 256, 0, stream>>>(residual, moe, out, n);
}

} // namespace ttl
