// prefill_ep.cu -- expert-parallel prefill: the token dispatch and the
// return of the experts' weighted outputs, around prefill.cu / prefill_tc.cu.
//
// Reference: GptOssModel::moe_batch, tt-lab src/model.cpp:340-461, split by
// expert owner.  Rank r holds its own tokens and experts [r*Ep, (r+1)*Ep)
// (Ep = E / world).  Per call:
//   router      on its own tokens (prefill.cu), replicated router weights;
//   plan        per destination rank d: which own tokens have an expert on d
//               (sent once each, in token order) and how many (token, expert)
//               pairs that is -- counts all-gathered so every rank knows every
//               send and receive size;
//   pack        the token rows and their top-4 (ids, weights) per destination;
//   dispatch    grouped NCCL send/recv (moe.cu);
//   experts     route / split / gate-up / down on the received tokens, whose
//               top-4 came with them (non-local experts are skipped);
//   return      per received token, in the sender's order, one row
//               w * down per local pair (the product rounded, as the
//               reference's combine rounds it), in rank order of the token's
//               top-4; grouped NCCL send/recv back to the owners;
//   combine     the owner adds its tokens' four rows in ascending expert id
//               (src/model.cpp:450-459), so the sum is the reference's.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace ttl {
namespace {

__device__ __forceinline__ int owner_of(int e, int per_rank) {
    return e / per_rank;
}

// One CTA per destination d: block scan over the own tokens in order.
// tok_off[t][d] = the token's send index to d (-1: none of its experts is
// on d); pair_off[t][d] = pairs to d of the tokens before it; cnt[d] tokens,
// cnt[world + d] pairs.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t *__restrict__ idx, int tokens, int world,
                                                       int per_rank, int32_t *tok_off, int32_t *pair_off,
                                                       int32_t *cnt) {
    __shared__ int warp_tok[32], warp_pair[32];
    const int d = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int base_tok = 0, base_pair = 0;
    for (int t0 = 0; t0 < tokens; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int np = 0;
        if (t < tokens) {
#pragma unroll
            for (int q = 0; q < kTopK; ++q) {
                const int e = idx[size_t(t) * 4 + q];
                np += (e >= 0 && owner_of(e, per_rank) == d) ? 1 : 0;
            }
        }
        const unsigned ballot = __ballot_sync(0xffffffffu, np > 0);
        int psum = np;  // inclusive warp scan of the pair counts
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, psum, o);
            psum += (lane >= o) ? v : 0;
        }
        if (lane == 31) {
            warp_tok[warp] = __popc(ballot);
            warp_pair[warp] = psum;
        }
        __syncthreads();
        int tok_before = 0, pair_before = 0, tok_total = 0, pair_total = 0;
        for (int k = 0; k < nwarps; ++k) {
            tok_before += k < warp ? warp_tok[k] : 0;
            pair_before += k < warp ? warp_pair[k] : 0;
            tok_total += warp_tok[k];
            pair_total += warp_pair[k];
        }
        if (t < tokens) {
            tok_off[size_t(t) * world + d] =
                np > 0 ? base_tok + tok_before + __popc(ballot & ((1u << lane) - 1u)) : -1;
            pair_off[size_t(t) * world + d] = base_pair + pair_before + psum - np;
        }
        base_tok += tok_total;
        base_pair += pair_total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        cnt[d] = base_tok;
        cnt[world + d] = base_pair;
    }
}

// One CTA per own token: its row and its top-4 into the send block of every
// destination it goes to.
__global__ void ep_pack_kernel(const float *__restrict__ x, const int32_t *__restrict__ idx,
                               const float *__restrict__ wts, int world, const int32_t *__restrict__ tok_off,
                               EpOffsets send_off, float *sendx, int32_t *send_idx, float *send_w) {
    const int t = blockIdx.x;
    for (int d = 0; d < world; ++d) {
        const int k = tok_off[size_t(t) * world + d];
        if (k < 0) {
            continue;
        }
        const size_t row = size_t(send_off.v[d]) + size_t(k);
        const float4 *src = reinterpret_cast<const float4 *>(x + size_t(t) * kDim);
        float4 *dst = reinterpret_cast<float4 *>(sendx + row * kDim);
        for (int i = threadIdx.x; i < kDim / 4; i += blockDim.x) {
            dst[i] = src[i];
        }
        if (threadIdx.x < kTopK) {
            send_idx[row * 4 + threadIdx.x] = idx[size_t(t) * 4 + threadIdx.x];
            send_w[row * 4 + threadIdx.x] = wts[size_t(t) * 4 + threadIdx.x];
        }
    }
}

// One CTA: ret_off[j] = local pairs of the received tokens before j (their
// rows in the return block, which is in receive order = the senders' order).
__global__ void __launch_bounds__(1024) ep_retoff_kernel(const int32_t *__restrict__ idx, int tokens, int rank,
                                                         int per_rank, int32_t *ret_off) {
    __shared__ int warp_pair[32];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int base = 0;
    for (int t0 = 0; t0 < tokens; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int np = 0;
        if (t < tokens) {
#pragma unroll
            for (int q = 0; q < kTopK; ++q) {
                const int e = idx[size_t(t) * 4 + q];
                np += (e >= 0 && owner_of(e, per_rank) == rank) ? 1 : 0;
            }
        }
        int psum = np;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, psum, o);
            psum += (lane >= o) ? v : 0;
        }
        if (lane == 31) {
            warp_pair[warp] = psum;
        }
        __syncthreads();
        int before = 0, total = 0;
        for (int k = 0; k < nwarps; ++k) {
            before += k < warp ? warp_pair[k] : 0;
            total += warp_pair[k];
        }
        if (t < tokens) {
            ret_off[t] = base + before + psum - np;
        }
        base += total;
        __syncthreads();
    }
}

// One CTA per received token j: its local pairs' rows w * down (rounded), in
// rank order of its top-4, at ret_off[j].
__global__ void ep_return_kernel(PrefillWork w, int rank, int per_rank, const int32_t *__restrict__ ret_off,
                                 float *ret) {
    const int j = blockIdx.x;
    int row = ret_off[j];
    for (int q = 0; q < kTopK; ++q) {
        const int e = w.top_idx[size_t(j) * 4 + q];
        if (e < 0 || owner_of(e, per_rank) != rank) {
            continue;
        }
        const int slot = w.pair_slot[size_t(j) * 4 + q];
        const float wt = w.top_w[size_t(j) * 4 + q];
        float *dst = ret + size_t(row) * kDim;
        if (slot >= 0) {
            const float *src = w.down + size_t(slot) * kDim;
            for (int i = threadIdx.x; i < kDim; i += blockDim.x) {
                dst[i] = __fmul_rn(wt, src[i]);
            }
        }
        ++row;
    }
}

// One CTA per own token: out = sum over its experts in ascending id of the
// returned rows w * down (src/model.cpp:450-459).  The row of (t, rank q) is
// in the block from e's owner d: back_off[d] + pair_off[t][d] + (pairs of t
// on d before q).
__global__ void ep_combine_kernel(const int32_t *__restrict__ idx, int world, int per_rank,
                                  const int32_t *__restrict__ pair_off, EpOffsets back_off,
                                  const float *__restrict__ back, float *out) {
    const int t = blockIdx.x;
    int e[4], rowq[4];
#pragma unroll
    for (int q = 0; q < kTopK; ++q) {
        e[q] = idx[size_t(t) * 4 + q];
    }
#pragma unroll
    for (int q = 0; q < kTopK; ++q) {
        const int d = owner_of(e[q], per_rank);
        int before = 0;
#pragma unroll
        for (int p = 0; p < kTopK; ++p) {
            before += (p < q && owner_of(e[p], per_rank) == d) ? 1 : 0;
        }
        rowq[q] = back_off.v[d] + pair_off[size_t(t) * world + d] + before;
    }
    // ascending expert id (the four ids are distinct)
    int order[4] = {0, 1, 2, 3};
#pragma unroll
    for (int i = 0; i < kTopK; ++i) {
#pragma unroll
        for (int k = 0; k + 1 < kTopK - i; ++k) {
            if (e[order[k]] > e[order[k + 1]]) {
                const int tmp = order[k];
                order[k] = order[k + 1];
                order[k + 1] = tmp;
            }
        }
    }
    for (int c = threadIdx.x; c < kDim; c += blockDim.x) {
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < kTopK; ++i) {
            o = __fadd_rn(o, back[size_t(rowq[order[i]]) * kDim + c]);
        }
        out[size_t(t) * kDim + c] = o;
    }
}

}  // namespace

void launch_ep_plan(const int32_t *idx, int tokens, int world, int per_rank, int32_t *tok_off, int32_t *pair_off,
                    int32_t *cnt, cudaStream_t stream) {
    ep_plan_kernel<<<world, 1024, 0, stream>>>(idx, tokens, world, per_rank, tok_off, pair_off, cnt);
}

void launch_ep_pack(const float *x, const int32_t *idx, const float *wts, int tokens, int world,
                    const int32_t *tok_off, const EpOffsets &send_off, float *sendx, int32_t *send_idx,
                    float *send_w, cudaStream_t stream) {
    ep_pack_kernel<<<tokens, 256, 0, stream>>>(x, idx, wts, world, tok_off, send_off, sendx, send_idx, send_w);
}

void launch_ep_return(const PrefillWork &w, int tokens, int rank, int per_rank, int32_t *ret_off, float *ret,
                      cudaStream_t stream) {
    ep_retoff_kernel<<<1, 1024, 0, stream>>>(w.top_idx, tokens, rank, per_rank, ret_off);
    ep_return_kernel<<<tokens, 256, 0, stream>>>(w, rank, per_rank, ret_off, ret);
}

void launch_ep_combine(const int32_t *idx, int tokens, int world, int per_rank, const int32_t *pair_off,
                       const EpOffsets &back_off, const float *back, float *out, cudaStream_t stream) {
    ep_combine_kernel<<<tokens, 256, 0, stream>>>(idx, world, per_rank, pair_off, back_off, back, out);
}

}  // namespace ttl
