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

constexpr int kRouterTokens = 8;          // tokens per router CTA
constexpr int kXRowStride = kDim + 4;     // padded shared row (bank spread)
constexpr int kGroup = 16;                // slots per expert-product group

__global__ void prefill_router_kernel(LayerDev L, PrefillWork w, int experts, int tokens,
                                      const float *__restrict__ x) {
    extern __shared__ float xs[];  // [kRouterTokens][kXRowStride]
    const int t0 = blockIdx.x * kRouterTokens;
    const int nt = min(kRouterTokens, tokens - t0);
    for (int i = threadIdx.x; i < nt * kDim; i += blockDim.x) {
        const int t = i / kDim;
        const int c = i - t * kDim;
        xs[t * kXRowStride + c] = x[size_t(t0 + t) * kDim + c];
    }
    __syncthreads();
    const int e = threadIdx.x / kRouterTokens;
    const int t = threadIdx.x % kRouterTokens;
    if (e >= experts || t >= nt) {
        return;
    }
    const float *wr = L.router_w + size_t(e) * kDim;
    const float *xr = xs + t * kXRowStride;
    float s = L.router_b[e];
    for (int c = 0; c < kDim; c += 8) {
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            p[j] = __fmul_rn(__ldg(wr + c + j), xr[c + j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s = __fadd_rn(s, p[j]);
        }
    }
    w.logits[size_t(t0 + t) * experts + e] = s;
}

__global__ void prefill_select_kernel(PrefillWork w, int experts, int tokens) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= tokens) {
        return;
    }
    const float *r = w.logits + size_t(t) * experts;
    uint8_t order[kMaxExperts];
    for (int i = 0; i < experts; ++i) {
        order[i] = uint8_t(i);
    }
    float sel[4];
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
        w.top_idx[t * 4 + i] = order[i];
        sel[i] = r[order[i]];
    }
    float maximum = -INFINITY;
    for (int i = 0; i < kTopK; ++i) {
        maximum = (maximum < sel[i]) ? sel[i] : maximum;
    }
    float wt[4];
    float sum = 0.0f;
    for (int i = 0; i < kTopK; ++i) {
        wt[i] = expf(__fsub_rn(sel[i], maximum));
        sum = __fadd_rn(sum, wt[i]);
    }
    for (int i = 0; i < kTopK; ++i) {
        w.top_w[t * 4 + i] = __fdiv_rn(wt[i], sum);
    }
}

// One CTA: histogram, offsets, stable buckets and the tile work list.
__global__ void __launch_bounds__(1024) prefill_route_kernel(PrefillWork w, int experts, int expert_begin,
                                                             int expert_count, int tokens) {
    __shared__ int counts[kMaxExperts];
    __shared__ int offsets[kMaxExperts + 1];
    for (int e = threadIdx.x; e < experts; e += blockDim.x) {
        counts[e] = 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tokens * kTopK; i += blockDim.x) {
        w.pair_slot[i] = -1;
        const int e = w.top_idx[i];
        if (e < 0 || e >= experts) {
            set_status(w.status, kStatusBadExpert);
            continue;
        }
        const int le = e - expert_begin;
        if (le >= 0 && le < expert_count) {
            atomicAdd(&counts[le], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        int tiles = 0;
        for (int le = 0; le < expert_count; ++le) {
            offsets[le] = run;
            w.counts[le] = counts[le];
            w.offsets[le] = run;
            for (int k = 0; k < counts[le]; k += kGroup) {
                w.tiles[tiles++] = (le << 20) | (run + k);
            }
            run += (counts[le] + kGroup - 1) / kGroup * kGroup;
        }
        offsets[expert_count] = run;
        w.offsets[expert_count] = run;
        *w.tile_count = tiles;
    }
    __syncthreads();
    // padding slots of each expert's last group
    for (int le = threadIdx.x; le < expert_count; le += blockDim.x) {
        for (int sl = offsets[le] + counts[le]; sl < offsets[le + 1]; ++sl) {
            w.pair_token[sl] = -1;
        }
    }
    // Stable placement: each warp owns experts; tokens are scanned in order.
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    for (int le = warp; le < expert_count; le += nwarps) {
        const int e = le + expert_begin;
        int base = offsets[le];
        for (int t0 = 0; t0 < tokens; t0 += 32) {
            const int t = t0 + lane;
            int rank = -1;
            if (t < tokens) {
#pragma unroll
                for (int r = 0; r < kTopK; ++r) {
                    if (w.top_idx[t * 4 + r] == e) {
                        rank = r;
                    }
                }
            }
            const unsigned ballot = __ballot_sync(0xffffffffu, rank >= 0);
            if (rank >= 0) {
                const int pos = base + __popc(ballot & ((1u << lane) - 1u));
                w.pair_token[pos] = t;
                w.pair_slot[t * 4 + rank] = pos;
            }
            base += __popc(ballot);
        }
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

void configure_prefill_kernels() {
    cudaFuncSetAttribute(prefill_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kRouterTokens * kXRowStride * int(sizeof(float)));
}

void launch_prefill_router(const LayerDev &L, const PrefillWork &w, const PrefillShape &s, const float *x,
                           cudaStream_t stream) {
    const int grid = (s.tokens + kRouterTokens - 1) / kRouterTokens;
    const int threads = s.experts * kRouterTokens;
    prefill_router_kernel<<<grid, threads, kRouterTokens * kXRowStride * sizeof(float), stream>>>(
        L, w, s.experts, s.tokens, x);
    prefill_select_kernel<<<(s.tokens + 127) / 128, 128, 0, stream>>>(w, s.experts, s.tokens);
}

void launch_prefill_route(const PrefillWork &w, const PrefillShape &s, cudaStream_t stream) {
    prefill_route_kernel<<<1, 1024, 0, stream>>>(w, s.experts, s.expert_begin, s.expert_count, s.tokens);
}

void launch_prefill_combine(const PrefillWork &w, const PrefillShape &s, float *out, cudaStream_t stream) {
    prefill_combine_kernel<<<s.tokens, 256, 0, stream>>>(w, s.tokens, out);
}

} // namespace ttl
