// prefill.cu -- batched (prefill) MoE: router, routing histogram and stable
// permute, grouped expert products, un-permute combine.
//
// Reference: GptOssModel::moe_batch, tt-lab src/model.cpp:340-461.
//   router      matmul_add_f32 (src/tensor.cpp:497-527): here one thread per
//               (token, expert) runs the reference's own sequential chain
//               (bias first, f32 products rounded, added in column order), so
//               logits -- and therefore top-4 indices -- equal the reference's
//               bit for bit.  Throughput-bound, so the exact order costs little.
//   top-4       selection sort + softmax per token (src/model.cpp:344-378).
//   histogram   per-expert counts, prefix offsets and buckets that are stable in
//               token order (src/model.cpp:380-394).
//   experts     grouped products over each expert's tokens (src/model.cpp:396-448)
//               with the SwiGLU epilogue (:423-433): tcgen05 block-scaled MMAs
//               in prefill_tc.cu, over groups of 16 slots (each expert's pairs
//               padded to a multiple of 16).
//   combine     per token, experts in ascending id order, out += w * down with
//               the product rounded first (src/model.cpp:450-459).
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ttl {
namespace {

constexpr int kRouterTokens = 4;                  // tokens per router CTA (one warp selects each)
constexpr int kRouterChunk = 64;                  // columns per staged chunk
constexpr int kRouterStages = 4;                  // chunks in flight
constexpr int kRouterRow = kRouterChunk + 4;      // padded shared row, floats (bank spread)
constexpr int kRouterChunks = kDim / kRouterChunk;  // 45
constexpr int kGroup = 16;                        // slots per expert-product group
static_assert(kDim % kRouterChunk == 0, "router chunks");

__host__ __device__ constexpr int router_threads(int experts) {
    return (experts * kRouterTokens + 31) / 32 * 32 < 32 * kRouterTokens ? 32 * kRouterTokens
                                                                       : (experts * kRouterTokens + 31) / 32 * 32;
}
__host__ __device__ constexpr size_t router_smem_bytes(int experts) {
    return (size_t(kRouterStages) * (experts + kRouterTokens) * kRouterRow + size_t(kRouterTokens) * kMaxExperts) *
               sizeof(float) +
           size_t(kRouterTokens) * kTopK * sizeof(int);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// The reference's selection sort (src/model.cpp:344-357): strict ">" over the
// permuted order the swaps leave, so ties and NaNs resolve as it does.
__device__ void select_sort_top4(const float *r, int experts, int idx[4]) {
    uint8_t order[kMaxExperts];
    for (int i = 0; i < experts; ++i) {
        order[i] = uint8_t(i);
    }
    for (int i = 0; i < kTopK; ++i) {
        int best = i;
        for (int j = i + 1; j < experts; ++j) {
            if (r[order[j]] > r[order[best]]) {
                best = j;
            }
        }
        const uint8_t tmp = order[i];
        order[i] = order[best];
        order[best] = tmp;
        idx[i] = order[i];
    }
}

// Router logits, top-4 and softmax for kRouterTokens tokens.  Thread (e, t)
// runs the reference's sequential chain for one logit (bias first, f32
// products rounded, added in column order), so logits -- and the indices --
// equal the reference's bit for bit.  Router rows and token rows stream
// through shared memory in 64-column chunks, kRouterStages in flight.
// Then warp t ranks token t's logits (larger first, lower index among equal
// values); when a NaN is present or a selected logit equals another expert's,
// the selection sort itself decides.
__global__ void prefill_router_kernel(LayerDev L, PrefillWork w, int experts, int tokens,
                                      const float *__restrict__ x) {
    extern __shared__ __align__(16) float rsm[];
    float *wst = rsm;                                                    // [stage][experts][kRouterRow]
    float *xst = wst + size_t(kRouterStages) * experts * kRouterRow;     // [stage][kRouterTokens][kRouterRow]
    float *lg = xst + kRouterStages * kRouterTokens * kRouterRow;        // [kRouterTokens][kMaxExperts]
    int *sel = reinterpret_cast<int *>(lg + kRouterTokens * kMaxExperts);  // [kRouterTokens][4]
    const int t0 = blockIdx.x * kRouterTokens;
    const int nt = min(kRouterTokens, tokens - t0);
    const int tid = threadIdx.x;
    const int per_chunk = (experts + nt) * (kRouterChunk / 4);

    auto issue = [&](int chunk) {
        const int st = chunk % kRouterStages;
        const int c0 = chunk * kRouterChunk;
        for (int i = tid; i < per_chunk; i += blockDim.x) {
            const int row = i / (kRouterChunk / 4);
            const int q = i - row * (kRouterChunk / 4);
            const float *src;
            float *dst;
            if (row < experts) {
                src = L.router_w + size_t(row) * kDim + c0 + 4 * q;
                dst = wst + (size_t(st) * experts + row) * kRouterRow + 4 * q;
            } else {
                const int t = row - experts;
                src = x + size_t(t0 + t) * kDim + c0 + 4 * q;
                dst = xst + (st * kRouterTokens + t) * kRouterRow + 4 * q;
            }
            cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(dst)), src);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    const int t = tid % kRouterTokens;
    const int e = tid / kRouterTokens;
    const bool active = e < experts && t < nt;
    float acc = active ? L.router_b[e] : 0.0f;
#pragma unroll
    for (int c = 0; c < kRouterStages - 1; ++c) {
        issue(c);
    }
    for (int c = 0; c < kRouterChunks; ++c) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kRouterStages - 2) : "memory");
        __syncthreads();
        if (c + kRouterStages - 1 < kRouterChunks) {
            issue(c + kRouterStages - 1);
        } else {
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        if (active) {
            const int st = c % kRouterStages;
            const float4 *wr = reinterpret_cast<const float4 *>(wst + (size_t(st) * experts + e) * kRouterRow);
            const float4 *xr = reinterpret_cast<const float4 *>(xst + (st * kRouterTokens + t) * kRouterRow);
#pragma unroll
            for (int j = 0; j < kRouterChunk / 4; ++j) {
                const float4 a = wr[j];
                const float4 b = xr[j];
                acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
                acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
                acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
                acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (active) {
        lg[t * kMaxExperts + e] = acc;
        w.logits[size_t(t0 + t) * experts + e] = acc;
    }
    __syncthreads();

    const int warp = tid >> 5;
    const int lane = tid & 31;
    if (warp >= nt) {
        return;
    }
    const float *r = lg + warp * kMaxExperts;
    float v[4];
    int rank[4];
    bool tie[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int ek = lane + 32 * k;
        v[k] = ek < experts ? r[ek] : 0.0f;
        rank[k] = 0;
        tie[k] = false;
    }
    bool amb = false;
    for (int j = 0; j < experts; ++j) {
        const float u = r[j];
        amb = amb | (u != u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int ek = lane + 32 * k;
            rank[k] += ((u > v[k]) | ((u == v[k]) & (j < ek))) ? 1 : 0;
            tie[k] = tie[k] | ((u == v[k]) & (j != ek));
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int ek = lane + 32 * k;
        if (ek < experts && rank[k] < kTopK) {
            sel[warp * kTopK + rank[k]] = ek;
            amb = amb | tie[k];
        }
    }
    amb = __any_sync(0xffffffffu, amb);
    __syncwarp();
    if (lane != 0) {
        return;
    }
    int idx[4];
    if (amb) {
        select_sort_top4(r, experts, idx);
    } else {
#pragma unroll
        for (int i = 0; i < kTopK; ++i) {
            idx[i] = sel[warp * kTopK + i];
        }
    }
    // softmax over the selected logits in rank order (src/model.cpp:358-378)
    const int tok = t0 + warp;
    float sv[4];
    float maximum = -INFINITY;
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        sv[i] = r[idx[i]];
        w.top_idx[tok * 4 + i] = idx[i];
        maximum = (maximum < sv[i]) ? sv[i] : maximum;
    }
    float wt[4];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        wt[i] = expf(__fsub_rn(sv[i], maximum));
        sum = __fadd_rn(sum, wt[i]);
    }
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        w.top_w[tok * 4 + i] = __fdiv_rn(wt[i], sum);
    }
}

__device__ __forceinline__ bool row_live(const PrefillWork &w, int t) {
    return !w.seg_count || t % w.seg_rows < w.seg_count[t / w.seg_rows];
}

// One CTA per local expert le (src/model.cpp:380-394): every CTA counts the
// routed pairs of all local experts (the same counts in every CTA), takes
// le's first slot, first group and first unit from the counts of the experts
// before it, writes le's groups, units and padding slots, and places le's
// pairs in its slots in token order (a block-wide scan over the tokens).
// Rows outside the live part of their segment (expert parallelism) are
// skipped.
// CTA 0 also writes the totals and marks pairs of experts that are not local.
__global__ void __launch_bounds__(1024) prefill_route_kernel(PrefillWork w, int experts, int expert_begin,
                                                             int expert_count, int tokens) {
    __shared__ int counts[kMaxExperts];
    __shared__ int warp_total[32];
    __shared__ int first[3];  // le's first slot, group and unit
    const int le = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (int e = threadIdx.x; e < expert_count; e += blockDim.x) {
        counts[e] = 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tokens * kTopK; i += blockDim.x) {
        if (!row_live(w, i / kTopK)) {
            if (le == 0) {
                w.pair_slot[i] = -1;
            }
            continue;
        }
        const int e = w.top_idx[i];
        const int l = e - expert_begin;
        if (e < 0 || e >= experts) {
            if (le == 0) {
                set_status(w.status, kStatusBadExpert);
                w.pair_slot[i] = -1;
            }
        } else if (l >= 0 && l < expert_count) {
            atomicAdd(&counts[l], 1);
        } else if (le == 0) {
            w.pair_slot[i] = -1;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0, groups = 0, units = 0;
        for (int l = 0; l < expert_count; ++l) {
            if (l == le) {
                first[0] = run;
                first[1] = groups;
                first[2] = units;
            }
            const int n = (counts[l] + kGroup - 1) / kGroup;
            run += n * kGroup;
            groups += n;
            units += (n + 1) / 2;
        }
        if (le == 0) {
            w.offsets[expert_count] = run;
            *w.tile_count = groups;
            *w.unit_count = units;
        }
    }
    __syncthreads();
    const int count = counts[le];
    const int n = (count + kGroup - 1) / kGroup;
    const int slot0 = first[0];
    if (threadIdx.x == 0) {
        w.counts[le] = count;
        w.offsets[le] = slot0;
    }
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        w.tiles[first[1] + k] = (le << 20) | (slot0 + k * kGroup);
        if ((k & 1) == 0) {
            w.units[first[2] + k / 2] = (first[1] + k) | (min(2, n - k) - 1) << 24;
        }
    }
    for (int sl = slot0 + count + threadIdx.x; sl < slot0 + n * kGroup; sl += blockDim.x) {
        w.pair_token[sl] = -1;  // padding slots of the last group
    }
    // stable placement: token order within the expert
    const int e = le + expert_begin;
    int base = slot0;
    for (int t0 = 0; t0 < tokens; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int rank = -1;
        if (t < tokens && row_live(w, t)) {
            const int4 q = *reinterpret_cast<const int4 *>(w.top_idx + size_t(t) * 4);
            rank = q.x == e ? 0 : q.y == e ? 1 : q.z == e ? 2 : q.w == e ? 3 : -1;
        }
        const unsigned ballot = __ballot_sync(0xffffffffu, rank >= 0);
        if (lane == 0) {
            warp_total[warp] = __popc(ballot);
        }
        __syncthreads();
        int before = 0, total = 0;
        for (int k = 0; k < int(blockDim.x >> 5); ++k) {
            const int c = warp_total[k];
            before += k < warp ? c : 0;
            total += c;
        }
        if (rank >= 0) {
            const int pos = base + before + __popc(ballot & ((1u << lane) - 1u));
            w.pair_token[pos] = t;
            w.pair_slot[t * 4 + rank] = pos;
        }
        base += total;
        __syncthreads();
    }
}

// out[t] = sum over the token's experts in ascending id of w * down.
__global__ void prefill_combine_kernel(PrefillWork w, int tokens, float *__restrict__ out) {
    const int t = blockIdx.x;
    if (t >= tokens) {
        return;
    }
    int e[4], r[4];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        e[i] = w.top_idx[t * 4 + i];
        r[i] = i;
    }
    // Sort the four (expert, rank) pairs by expert id (distinct ids).
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
#pragma unroll
        for (int j = 0; j + 1 < kTopK - i; ++j) {
            if (e[j] > e[j + 1]) {
                const int te = e[j], tr = r[j];
                e[j] = e[j + 1];
                r[j] = r[j + 1];
                e[j + 1] = te;
                r[j + 1] = tr;
            }
        }
    }
    int slot[4];
    float wt[4];
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
        slot[i] = w.pair_slot[t * 4 + r[i]];
        wt[i] = w.top_w[t * 4 + r[i]];
    }
    for (int c = threadIdx.x; c < kDim; c += blockDim.x) {
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < kTopK; ++i) {
            if (slot[i] >= 0) {
                o = __fadd_rn(o, __fmul_rn(wt[i], w.down[size_t(slot[i]) * kDim + c]));
            }
        }
        out[size_t(t) * kDim + c] = o;
    }
}

} // namespace

// The prefill kernels alternate with the tensor-core kernels (about 200 KB
// of shared memory each) on one stream: every kernel asks for the largest
// shared-memory carveout, so no launch waits for the SMs to repartition L1.
void configure_prefill_kernels() {
    cudaFuncSetAttribute(prefill_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(router_smem_bytes(kMaxExperts)));
    cudaFuncSetAttribute(prefill_router_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    cudaFuncSetAttribute(prefill_route_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    cudaFuncSetAttribute(prefill_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
}

void launch_prefill_router(const LayerDev &L, const PrefillWork &w, const PrefillShape &s, const float *x,
                           cudaStream_t stream) {
    const int grid = (s.tokens + kRouterTokens - 1) / kRouterTokens;
    prefill_router_kernel<<<grid, router_threads(s.experts), router_smem_bytes(s.experts), stream>>>(
        L, w, s.experts, s.tokens, x);
}

void launch_prefill_route(const PrefillWork &w, const PrefillShape &s, cudaStream_t stream) {
    prefill_route_kernel<<<s.expert_count, 1024, 0, stream>>>(w, s.experts, s.expert_begin, s.expert_count,
                                                               s.tokens);
}

void launch_prefill_combine(const PrefillWork &w, const PrefillShape &s, float *out, cudaStream_t stream) {
    prefill_combine_kernel<<<s.tokens, 256, 0, stream>>>(w, s.tokens, out);
}

} // namespace ttl
