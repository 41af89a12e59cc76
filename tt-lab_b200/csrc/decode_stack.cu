// decode_stack.cu -- persistent decode kernel: every token x layer of a decode
// call in one cooperative launch (one CTA per SM).
//
// Reference: GptOssModel::moe (tt-lab src/model.cpp:292-338) and the per-layer
// RMSNorm -> moe -> residual sequence of GptOssModel::forward
// (src/model.cpp:590-594).
//
// Per layer the grid meets at two bounded grid barriers:
//   A  select:  every CTA reads the layer's router sums, forms the logits and
//               picks the same top 4 (no exchange needed); h = RMSNorm(x)*w
//               goes to shared memory.
//   B  gate/up: the (selected expert, row) pairs are split evenly over all
//               warps; each warp streams the gate and up rows as 16-byte
//               vectors (lanes split K, loads for the next row issued before
//               the current row is computed), applies the block scales, and
//               writes SwiGLU(gate, up) to `hidden`.  Meanwhile each CTA
//               prefetches into L2 the down-projection rows it will need in C
//               (cp.async.bulk.prefetch.L2), so HBM streams both phases' bytes
//               back to back.
//   -- barrier --
//   C  down:    each CTA owns a contiguous slice of output rows; warps compute
//               the four experts' rows from L2, combine in rank order, add the
//               residual, and (stack mode) accumulate the NEXT layer's router
//               sums for their rows -- the RMSNorm scale is a scalar, so
//               logit_e = b_e + s * sum_c W_ec g_c x_c splits over row slices --
//               with f64 atomics.
//   -- barrier --
// Mode 0 (single layer, h given): the logits come from a router phase instead
// (CTA e < E computes expert e's logit and a bound on the reference's own f32
// summation error); if any selected logit's interval touches another expert's,
// the candidates are re-evaluated exactly in the reference's order, so the
// indices equal the reference's bit for bit.
//
// Every wait is bounded (about 2 s); on timeout the kernel sets
// kStatusWaitTimeout and returns, and ttl_moe_sync reports TTL_ERR_DEVICE.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ttl {
namespace {

constexpr int kThreads = 384;
constexpr int kWarps = kThreads / 32;
constexpr int kXStride = 36;                        // padded floats per K-block
constexpr int kVec = kBlocks * kXStride;            // one padded 2880-vector
constexpr unsigned long long kSpinLimit = 1ull << 26;
constexpr int kColsPerWarp = kDim / kWarps;           // router columns per warp (mode 0)
constexpr int kColsPerLane = (kColsPerWarp + 31) / 32;
static_assert(kDim % kWarps == 0, "router column split");

struct Smem {
    float h[kVec];               // expert input of the current layer
    float hid[kTopK][kVec];      // hidden vectors for the down phase
    float logit[kMaxExperts];
    float bound[kMaxExperts];
    float val[kMaxExperts];
    double red[kWarps];
    int sel[kTopK];              // selected experts, rank order
    int local[kTopK];            // local index or -1
    float wts[kTopK];
    int n_local;                 // selected experts owned here
    int slot_of[kTopK];          // compact slot -> rank
    int amb;
    int abort;
    float scale;                 // RMSNorm scale of the current layer
};

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float ld_cg(const float *p) {
    return __ldcg(p);
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Dot of one 32-element block (16 packed bytes) with xs[0..31] (f32 exact E2M1).
__device__ __forceinline__ float block_dot(const uint4 q, const float *xb) {
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int wd = 0; wd < 4; ++wd) {
        const float4 xa = *reinterpret_cast<const float4 *>(xb + wd * 8);
        const float4 xc = *reinterpret_cast<const float4 *>(xb + wd * 8 + 4);
        const float2 v0 = __half22float2(e2m1x2_to_half2(words[wd] & 0xffu));
        const float2 v1 = __half22float2(e2m1x2_to_half2((words[wd] >> 8) & 0xffu));
        const float2 v2 = __half22float2(e2m1x2_to_half2((words[wd] >> 16) & 0xffu));
        const float2 v3 = __half22float2(e2m1x2_to_half2(words[wd] >> 24));
        a0 = fmaf(v0.x, xa.x, a0);
        a1 = fmaf(v0.y, xa.y, a1);
        a0 = fmaf(v1.x, xa.z, a0);
        a1 = fmaf(v1.y, xa.w, a1);
        a0 = fmaf(v2.x, xc.x, a0);
        a1 = fmaf(v2.y, xc.y, a1);
        a0 = fmaf(v3.x, xc.z, a0);
        a1 = fmaf(v3.y, xc.w, a1);
    }
    return a0 + a1;
}

// Bounded grid barrier.  bar[0] counts arrivals, bar[1] is the generation.
__device__ bool grid_barrier(unsigned *bar, unsigned &gen, uint32_t *status, Smem &s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned arrived = atomicAdd(&bar[0], 1u);
        if (arrived == gridDim.x - 1) {
            bar[0] = 0u;
            __threadfence();
            atomicExch(&bar[1], gen + 1u);
        } else {
            unsigned long long spins = 0;
            unsigned cur;
            do {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(bar + 1) : "memory");
                if (cur != gen) {
                    break;
                }
                if (++spins > kSpinLimit) {
                    set_status(status, kStatusWaitTimeout);
                    s.abort = 1;
                    break;
                }
                __nanosleep(32);
            } while (true);
        }
        gen += 1u;
        __threadfence();
    }
    __syncthreads();
    return s.abort == 0;
}

__device__ __forceinline__ double block_sum_d(double v, Smem &s) {
    v = warp_sum_d(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        s.red[threadIdx.x >> 5] = v;
    }
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) {
        t += s.red[i];
    }
    return t;
}

// Loads a 2880-vector (written by this kernel: bypass L1) into padded smem.
__device__ __forceinline__ void load_vec_cg(float *dst, const float *src) {
    for (int i = threadIdx.x; i < kDim / 4; i += kThreads) {
        const float4 q = __ldcg(reinterpret_cast<const float4 *>(src) + i);
        *reinterpret_cast<float4 *>(dst + ((4 * i) >> 5) * kXStride + ((4 * i) & 31)) = q;
    }
}

__device__ void select_top4_ref(const float *vals, int experts, int idx[4]) {
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

__device__ float exact_logit(const float *__restrict__ wrow, float bias, const float *hpad) {
    float acc = bias;
    for (int c = 0; c < kDim; c += 8) {
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = c + j;
            p[j] = __fmul_rn(__ldg(wrow + k), hpad[(k >> 5) * kXStride + (k & 31)]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            acc = __fadd_rn(acc, p[j]);
        }
    }
    return acc;
}

// Warp 0: top 4 of s.logit by value (lowest index on exact ties); flags
// ambiguity when `check_bounds` and an interval of a selected expert touches
// another expert's.
__device__ void warp_top4(Smem &s, int experts, bool check_bounds) {
    const int lane = threadIdx.x & 31;
    int chosen[4];
    bool invalid = false;
    for (int r = 0; r < kTopK; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = lane; i < experts; i += 32) {
            bool taken = false;
            for (int q = 0; q < r; ++q) {
                taken |= (chosen[q] == i);
            }
            const float v = s.logit[i];
            if (!taken && (bi == 0x7fffffff || v > bv || (v == bv && i < bi))) {
                bv = v;
                bi = i;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi == 0x7fffffff || !(bv == bv)) {
            invalid = true;
            bi = r;
        }
        chosen[r] = bi;
    }
    bool amb = invalid;
    if (check_bounds) {
        for (int i = lane; i < experts; i += 32) {
            for (int q = 0; q < kTopK; ++q) {
                const int a = chosen[q];
                if (a != i && !(fabsf(s.logit[a] - s.logit[i]) > s.bound[a] + s.bound[i])) {
                    amb = true;
                }
            }
        }
    }
    amb = __any_sync(0xffffffffu, amb);
    if (lane == 0) {
        s.amb = amb ? 1 : 0;
        for (int q = 0; q < kTopK; ++q) {
            s.sel[q] = chosen[q];
        }
    }
}

__device__ void finish_selection(Smem &s, const StackArgs &a) {
    // softmax (src/model.cpp:310-321) and local ownership
    if (threadIdx.x == 0) {
        float maximum = -INFINITY;
        float v[4], w[4];
        for (int q = 0; q < kTopK; ++q) {
            v[q] = s.val[s.sel[q]];
            maximum = (maximum < v[q]) ? v[q] : maximum;
        }
        float sum = 0.0f;
        for (int q = 0; q < kTopK; ++q) {
            w[q] = expf(__fsub_rn(v[q], maximum));
            sum = __fadd_rn(sum, w[q]);
        }
        int n = 0;
        for (int q = 0; q < kTopK; ++q) {
            s.wts[q] = __fdiv_rn(w[q], sum);
            const int le = s.sel[q] - a.expert_begin;
            s.local[q] = (le >= 0 && le < a.expert_count) ? le : -1;
            if (s.local[q] >= 0) {
                s.slot_of[n++] = q;
            }
        }
        s.n_local = n;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) decode_stack_kernel(StackArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem &s = *reinterpret_cast<Smem *>(smem_raw);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nblk = gridDim.x;
    const int E = a.experts;
    unsigned gen = 0;
    if (threadIdx.x == 0) {
        s.abort = 0;
        gen = *reinterpret_cast<volatile unsigned *>(a.barrier + 1);
    }
    __syncthreads();

    // Output rows of this CTA in phase C (and its router-sum rows).
    const int r0 = int((long long)blockIdx.x * kDim / nblk);
    const int r1 = int((long long)(blockIdx.x + 1) * kDim / nblk);
    const int nl = a.layer_end - a.layer_begin;

    // Router sums of (token 0, first layer) in stack mode.
    if (a.mode == 1) {
        const StackLayer &L = a.layers[a.layer_begin];
        double *acc = a.acc;  // parity 0
        const float *x = a.x;
        for (int e = warp; e < E + 1; e += kWarps) {
            const int r = r0 + lane;
            double v = 0.0;
            if (r < r1) {
                const float xr = x[r];
                v = (e < E) ? double(__ldg(L.router_w + size_t(e) * kDim + r)) * double(__fmul_rn(xr, L.norm_w[r]))
                            : double(__fmul_rn(xr, xr));
            }
            v = warp_sum_d(v);
            if (lane == 0) {
                atomicAdd(acc + e, v);
            }
        }
    }
    if (!grid_barrier(a.barrier, gen, a.status, s)) {
        return;
    }

    for (int t = 0; t < a.tokens; ++t) {
        for (int li = 0; li < nl; ++li) {
            const int l = a.layer_begin + li;
            const StackLayer &L = a.layers[l];
            const int step = t * nl + li;
            const float *xcur = (li == 0) ? a.x + size_t(t) * kDim : a.y + size_t(t) * kDim;
            float *ycur = a.y + size_t(t) * kDim;

            // ---------------- A: selection ----------------
            if (a.mode == 1) {
                const double *acc = a.acc + size_t(step & 1) * (kMaxExperts + 1);
                if (threadIdx.x == 0) {
                    const float ss = float(__ldcg(acc + E));
                    s.scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(kDim)), 1.0e-5f)));
                }
                __syncthreads();
                for (int e = threadIdx.x; e < E; e += kThreads) {
                    const double p = __ldcg(acc + e);
                    const float lg = float(double(L.router_b[e]) + double(s.scale) * p);
                    s.logit[e] = lg;
                    s.val[e] = lg;
                }
                // h = (x * scale) * w
                for (int i = threadIdx.x; i < kDim; i += kThreads) {
                    const float xv = ld_cg(xcur + i);
                    s.h[(i >> 5) * kXStride + (i & 31)] = __fmul_rn(__fmul_rn(xv, s.scale), L.norm_w[i]);
                }
                // the other accumulator parity is zeroed for the layer after next
                if (blockIdx.x == 0) {
                    double *other = a.acc + size_t((step + 1) & 1) * (kMaxExperts + 1);
                    // it was read during the previous layer's A phase, which every
                    // CTA finished before the barrier that ended its C phase
                    for (int e = threadIdx.x; e < E + 1; e += kThreads) {
                        other[e] = 0.0;
                    }
                }
                __syncthreads();
                if (warp == 0) {
                    warp_top4(s, E, false);
                }
                __syncthreads();
            } else {
                // h given; CTA e < E computes expert e's logit and error bound.
                for (int i = threadIdx.x; i < kDim / 4; i += kThreads) {
                    const float4 q = __ldcg(reinterpret_cast<const float4 *>(xcur) + i);
                    *reinterpret_cast<float4 *>(s.h + ((4 * i) >> 5) * kXStride + ((4 * i) & 31)) = q;
                }
                __syncthreads();
                for (int e = blockIdx.x; e < E; e += nblk) {
                    const float *wr = L.router_w + size_t(e) * kDim;
                    // Each warp owns a contiguous chunk of columns and each lane a
                    // contiguous run inside it, so prefix sums follow column order;
                    // the exact prefix sums give the bound u * sum |s_c|.
                    const int c0 = warp * kColsPerWarp;
                    double loc = 0.0;
                    float p[kColsPerLane];
#pragma unroll
                    for (int j = 0; j < kColsPerLane; ++j) {
                        const int off = lane * kColsPerLane + j;
                        const int c = c0 + off;
                        p[j] = (off < kColsPerWarp) ? __fmul_rn(__ldg(wr + c), s.h[(c >> 5) * kXStride + (c & 31)])
                                                    : 0.0f;
                        loc += double(p[j]);
                    }
                    double inc = loc;
                    for (int o = 1; o < 32; o <<= 1) {
                        const double tt = __shfl_up_sync(0xffffffffu, inc, o);
                        if (lane >= o) {
                            inc += tt;
                        }
                    }
                    __syncthreads();
                    if (lane == 31) {
                        s.red[warp] = inc;
                    }
                    __syncthreads();
                    double base = double(L.router_b[e]);
                    for (int i = 0; i < warp; ++i) {
                        base += s.red[i];
                    }
                    double run = base + inc - loc;
                    double abs_sum = 0.0;
#pragma unroll
                    for (int j = 0; j < kColsPerLane; ++j) {
                        run += double(p[j]);
                        abs_sum += fabs(run);
                    }
                    double total = 0.0;
                    for (int i = 0; i < kWarps; ++i) {
                        total += s.red[i];
                    }
                    const double abs_total = block_sum_d(abs_sum, s);
                    if (threadIdx.x == 0) {
                        const double logit = double(L.router_b[e]) + total;
                        a.logits[e] = float(logit);
                        a.bounds[e] = float((1.02 * 5.9604644775390625e-08 * abs_total +
                                             5.9604644775390625e-08 * fabs(logit) + 1e-30) * 1.0001);
                    }
                    __syncthreads();
                }
                if (!grid_barrier(a.barrier, gen, a.status, s)) {
                    return;
                }
                for (int e = threadIdx.x; e < E; e += kThreads) {
                    s.logit[e] = __ldcg(a.logits + e);
                    s.bound[e] = __ldcg(a.bounds + e);
                    s.val[e] = s.logit[e];
                }
                __syncthreads();
                if (warp == 0) {
                    warp_top4(s, E, true);
                }
                __syncthreads();
                if (s.amb) {
                    float lower = INFINITY;
                    for (int q = 0; q < kTopK; ++q) {
                        lower = fminf(lower, s.logit[s.sel[q]] - s.bound[s.sel[q]]);
                    }
                    for (int e = threadIdx.x; e < E; e += kThreads) {
                        if (!(s.logit[e] + s.bound[e] < lower)) {
                            s.val[e] = exact_logit(L.router_w + size_t(e) * kDim, L.router_b[e], s.h);
                        }
                    }
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        int idx[4];
                        select_top4_ref(s.val, E, idx);
                        for (int q = 0; q < kTopK; ++q) {
                            s.sel[q] = idx[q];
                        }
                        if (blockIdx.x == 0) {
                            atomicAdd(&a.counters[0], 1ull);
                        }
                    }
                    __syncthreads();
                }
            }
            finish_selection(s, a);
            if (blockIdx.x == 0 && threadIdx.x < kTopK && t == a.tokens - 1 && li == nl - 1) {
                a.top_idx[threadIdx.x] = s.sel[threadIdx.x];
                a.top_w[threadIdx.x] = s.wts[threadIdx.x];
            }

            // ---------------- B: gate/up + SwiGLU ----------------
            const int n_items = s.n_local * kDim;
            if (threadIdx.x < s.n_local * 2) {
                // L2 prefetch of this CTA's down rows for phase C (nibbles, scales)
                const int q = s.slot_of[threadIdx.x >> 1];
                const uint8_t *m = L.down + size_t(s.local[q]) * kPackedMatrixBytes;
                if ((threadIdx.x & 1) == 0) {
                    prefetch_l2(m + size_t(r0) * kNibbleRowBytes, uint32_t((r1 - r0) * kNibbleRowBytes));
                } else {
                    const size_t lo = scale_block_offset(r0 >> 7, 0);
                    const size_t hi = scale_block_offset(((r1 - 1) >> 7) + 1, 0);
                    prefetch_l2(m + lo, uint32_t(hi - lo));
                }
            }
            {
                const int i0 = int((long long)blockIdx.x * n_items / nblk);
                const int i1 = int((long long)(blockIdx.x + 1) * n_items / nblk);
                int item = i0 + warp;
                uint4 gq[3], uq[3];
                uint32_t gs[3], us[3];
                auto load = [&](int it) {
                    const int slot = it / kDim;
                    const int row = it - slot * kDim;
                    const int le = s.local[s.slot_of[slot]];
                    const uint8_t *gm = L.gate + size_t(le) * kPackedMatrixBytes;
                    const uint8_t *um = L.up + size_t(le) * kPackedMatrixBytes;
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        const int kb = lane + 32 * j;
                        if (kb < kBlocks) {
                            gq[j] = ldg_stream(gm + size_t(row) * kNibbleRowBytes + kb * 16);
                            uq[j] = ldg_stream(um + size_t(row) * kNibbleRowBytes + kb * 16);
                            gs[j] = __ldg(gm + scale_offset(row, kb));
                            us[j] = __ldg(um + scale_offset(row, kb));
                        }
                    }
                };
                if (item < i1) {
                    load(item);
                }
                while (item < i1) {
                    uint4 cg[3], cu[3];
                    uint32_t cgs[3], cus[3];
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        cg[j] = gq[j];
                        cu[j] = uq[j];
                        cgs[j] = gs[j];
                        cus[j] = us[j];
                    }
                    const int cur = item;
                    item += kWarps;
                    if (item < i1) {
                        load(item);  // next row's loads are in flight during this row's math
                    }
                    float ag = 0.0f, au = 0.0f;
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        const int kb = lane + 32 * j;
                        if (kb < kBlocks) {
                            const float *xb = s.h + kb * kXStride;
                            ag = fmaf(e8m0_ref_scale(cgs[j]), 2.0f * block_dot(cg[j], xb), ag);
                            au = fmaf(e8m0_ref_scale(cus[j]), 2.0f * block_dot(cu[j], xb), au);
                        }
                    }
                    ag = warp_sum(ag);
                    au = warp_sum(au);
                    if (lane == 0) {
                        const int slot = cur / kDim;
                        const int row = cur - slot * kDim;
                        const int le = s.local[s.slot_of[slot]];
                        const float g = __fadd_rn(L.gate_b[size_t(le) * kDim + row], ag);
                        const float u = __fadd_rn(L.up_b[size_t(le) * kDim + row], au);
                        a.hidden[size_t(slot) * kDim + row] = swiglu_ref(g, u);
                    }
                }
            }
            if (!grid_barrier(a.barrier, gen, a.status, s)) {
                return;
            }

            // ---------------- C: down + combine + residual ----------------
            {
                const int nloc = s.n_local;
                // issue this warp's first row loads before staging `hidden`
                const int rows = r1 - r0;
                uint4 q[kTopK][3];
                uint32_t sb[kTopK][3];
                auto load_row = [&](int row) {
#pragma unroll
                    for (int k = 0; k < kTopK; ++k) {
                        if (k < nloc) {
                            const uint8_t *m = L.down + size_t(s.local[s.slot_of[k]]) * kPackedMatrixBytes;
#pragma unroll
                            for (int j = 0; j < 3; ++j) {
                                const int kb = lane + 32 * j;
                                if (kb < kBlocks) {
                                    q[k][j] = *reinterpret_cast<const uint4 *>(m + size_t(row) * kNibbleRowBytes + kb * 16);
                                    sb[k][j] = m[scale_offset(row, kb)];
                                }
                            }
                        }
                    }
                };
                if (warp < rows) {
                    load_row(r0 + warp);
                }
                for (int k = 0; k < nloc; ++k) {
                    load_vec_cg(s.hid[k], a.hidden + size_t(k) * kDim);
                }
                __syncthreads();
                for (int rr = warp; rr < rows; rr += kWarps) {
                    const int row = r0 + rr;
                    if (rr != warp) {
                        load_row(row);
                    }
                    float acc[kTopK];
#pragma unroll
                    for (int k = 0; k < kTopK; ++k) {
                        float v = 0.0f;
                        if (k < nloc) {
#pragma unroll
                            for (int j = 0; j < 3; ++j) {
                                const int kb = lane + 32 * j;
                                if (kb < kBlocks) {
                                    v = fmaf(e8m0_ref_scale(sb[k][j]),
                                             2.0f * block_dot(q[k][j], s.hid[k] + kb * kXStride), v);
                                }
                            }
                        }
                        acc[k] = warp_sum(v);
                    }
                    if (lane == 0) {
                        // combine in rank order (src/model.cpp:323, :333-336)
                        float o = 0.0f;
                        for (int rank = 0; rank < kTopK; ++rank) {
                            int k = -1;
                            for (int j = 0; j < nloc; ++j) {
                                if (s.slot_of[j] == rank) {
                                    k = j;
                                }
                            }
                            if (k >= 0) {
                                const int le = s.local[rank];
                                const float d = __fadd_rn(L.down_b[size_t(le) * kDim + row], acc[k]);
                                o = __fadd_rn(o, __fmul_rn(s.wts[rank], d));
                            }
                        }
                        ycur[row] = (a.mode == 1) ? __fadd_rn(ld_cg(xcur + row), o) : o;
                    }
                }
                // stack mode: router sums of the next (token, layer) over this CTA's rows
                if (a.mode == 1) {
                    const bool more_layers = (li + 1 < nl);
                    const bool more_tokens = (t + 1 < a.tokens);
                    if (more_layers || more_tokens) {
                        __syncthreads();  // this CTA's y rows are written
                        const StackLayer &N = a.layers[more_layers ? l + 1 : a.layer_begin];
                        const float *xn = more_layers ? ycur : a.x + size_t(t + 1) * kDim;
                        double *acc = a.acc + size_t((step + 1) & 1) * (kMaxExperts + 1);
                        for (int e = warp; e < E + 1; e += kWarps) {
                            const int r = r0 + lane;
                            double v = 0.0;
                            if (r < r1) {
                                const float xr = ld_cg(xn + r);
                                v = (e < E) ? double(__ldg(N.router_w + size_t(e) * kDim + r)) *
                                                  double(__fmul_rn(xr, N.norm_w[r]))
                                            : double(__fmul_rn(xr, xr));
                            }
                            v = warp_sum_d(v);
                            if (lane == 0) {
                                atomicAdd(acc + e, v);
                            }
                        }
                    }
                }
            }
            if (!grid_barrier(a.barrier, gen, a.status, s)) {
                return;
            }
        }
    }
}

} // namespace

size_t stack_smem_bytes() {
    return sizeof(Smem);
}

void configure_stack_kernel() {
    cudaFuncSetAttribute(decode_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(Smem)));
}

cudaError_t launch_decode_stack(const StackArgs &args, int sms, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = sizeof(Smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_stack_kernel, args);
}

} // namespace ttl
