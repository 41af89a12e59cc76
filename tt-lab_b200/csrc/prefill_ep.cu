// prefill_ep.cu -- expert-parallel prefill over peer memory: the token
// dispatch to the experts' owners and the return of their weighted outputs,
// around prefill.cu / prefill_tc.cu, with no host round trip and no NCCL.
//
// Reference: GptOssModel::moe_batch, tt-lab src/model.cpp:340-461, split by
// expert owner.  Rank r holds its own tokens and experts [r*Ep, (r+1)*Ep)
// (Ep = E / world).  Every rank owns a receive block (EpInbox, an IPC
// allocation every peer maps over NVLink).  Per call, with a call tag agreed
// by all ranks:
//   router   on its own tokens (prefill.cu), replicated router weights;
//   plan     per destination d: which own tokens have an expert on d (each
//            sent once, in token order: its row index in d's region for this
//            rank) and how many;
//   send     each token's row, top-4 and own index written straight into the
//            region of this rank in every destination's block (peer stores);
//            the last CTA, after a system fence, publishes the tagged row
//            counts;
//   wait     the receiver polls the tagged counts of all sources (bounded);
//   experts  route / split / gate-up / down over [world][cap] rows, the dead
//            tail of each source's region skipped (PrefillWork::seg_count);
//   back     per live received row and local pair, w * down (the product
//            rounded, as the reference's combine rounds it) written into the
//            source's block at (token, rank q); then tagged done flags;
//   combine  the owner waits for every rank's done flag (bounded) and adds
//            its tokens' four rows in ascending expert id
//            (src/model.cpp:450-459), so the sum is the reference's.
// Ordering between calls: a rank starts call n+1 only after every rank's
// done flag of call n, i.e. after every peer has finished reading its block
// for call n, so rows of n+1 never overwrite rows still in use.
// A missing peer ends the waits after 2 s with kStatusWaitTimeout.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace ttl {
namespace {

__device__ __forceinline__ int owner_of(int e, int per_rank) {
    return e / per_rank;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long tagged_word(uint32_t tag, uint32_t v) {
    return (static_cast<unsigned long long>(tag) << 32) | v;
}

// The last CTA to arrive (after every CTA's system-scope fence) publishes
// `word(d)` into flags[rank] of every rank's block: the peer that acquires
// the flag sees every row this grid wrote into its block.
template <class F>
__device__ __forceinline__ void publish_last(const EpPeers &peers, int world, int cap, int rank, bool done_flag,
                                             unsigned *arrive, F word) {
    __threadfence_system();
    __syncthreads();
    __shared__ unsigned last;
    if (threadIdx.x == 0) {
        last = atomicAdd(arrive, 1u) == gridDim.x - 1 ? 1u : 0u;
    }
    __syncthreads();
    if (last && threadIdx.x < world) {
        __threadfence_system();
        const int d = threadIdx.x;
        EpInbox in = ep_inbox_at(peers.base[d], world, cap);
        unsigned long long *flag = (done_flag ? in.done : in.cnt) + rank;
        asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(flag), "l"(word(d)) : "memory");
    }
}

// One CTA per destination d: block scan over the own tokens in order.
// tok_off[t][d] = the token's row in d's region for this rank (-1: none of
// its experts is on d); cnt[d] = rows sent to d.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t *__restrict__ idx, int tokens, int world,
                                                       int per_rank, int32_t *tok_off, int32_t *cnt) {
    __shared__ int warp_tok[32];
    const int d = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    int base_tok = 0;
    for (int t0 = 0; t0 < tokens; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        bool to_d = false;
        if (t < tokens) {
#pragma unroll
            for (int q = 0; q < kTopK; ++q) {
                const int e = idx[size_t(t) * 4 + q];
                to_d = to_d || (e >= 0 && owner_of(e, per_rank) == d);
            }
        }
        const unsigned ballot = __ballot_sync(0xffffffffu, to_d);
        if (lane == 0) {
            warp_tok[warp] = __popc(ballot);
        }
        __syncthreads();
        int before = 0, total = 0;
        for (int k = 0; k < nwarps; ++k) {
            before += k < warp ? warp_tok[k] : 0;
            total += warp_tok[k];
        }
        if (t < tokens) {
            tok_off[size_t(t) * world + d] = to_d ? base_tok + before + __popc(ballot & ((1u << lane) - 1u)) : -1;
        }
        base_tok += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        cnt[d] = base_tok;
    }
}

// CTAs stride over the own tokens: each token's row, top-4 and index go to
// this rank's region in every destination's block (peer stores over NVLink,
// 16 B each); then the tagged row counts.
__global__ void __launch_bounds__(256) ep_send_kernel(const float *__restrict__ x, const int32_t *__restrict__ idx,
                                                      const float *__restrict__ wts, int tokens, int world,
                                                      int rank, int cap, const int32_t *__restrict__ tok_off,
                                                      const int32_t *__restrict__ cnt, EpPeers peers, uint32_t tag,
                                                      unsigned *arrive) {
    for (int t = blockIdx.x; t < tokens; t += gridDim.x) {
        const float4 *src = reinterpret_cast<const float4 *>(x + size_t(t) * kDim);
        for (int d = 0; d < world; ++d) {
            const int k = tok_off[size_t(t) * world + d];
            if (k < 0) {
                continue;
            }
            EpInbox in = ep_inbox_at(peers.base[d], world, cap);
            const size_t row = size_t(rank) * cap + size_t(k);
            float4 *dst = reinterpret_cast<float4 *>(in.x + row * kDim);
            for (int i = threadIdx.x; i < kDim / 4; i += blockDim.x) {
                dst[i] = src[i];
            }
            if (threadIdx.x < kTopK) {
                in.idx[row * 4 + threadIdx.x] = idx[size_t(t) * 4 + threadIdx.x];
                in.w[row * 4 + threadIdx.x] = wts[size_t(t) * 4 + threadIdx.x];
            } else if (threadIdx.x == kTopK) {
                in.src[row] = t;
            }
        }
    }
    publish_last(peers, world, cap, rank, false, arrive,
                 [&](int d) { return tagged_word(tag, uint32_t(cnt[d])); });
}

// One warp: lane d polls flags[d] (system scope, acquire) until it carries
// `tag`, for at most 2 s; counts[d] = its value clamped to cap (0 on a
// timeout, with kStatusWaitTimeout; kStatusCapacity when above cap).
__global__ void ep_wait_kernel(const unsigned long long *flags, int world, uint32_t tag, int cap, int32_t *counts,
                               uint32_t *status) {
    const int d = threadIdx.x;
    if (d >= world) {
        return;
    }
    unsigned long long w = 0;
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
        asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(flags + d) : "memory");
        if (uint32_t(w >> 32) == tag) {
            break;
        }
        if (globaltimer_ns() - t0 > 2000000000ull) {
            set_status(status, kStatusWaitTimeout);
            w = 0;
            break;
        }
    }
    if (counts) {
        uint32_t n = uint32_t(w);
        if (n > uint32_t(cap)) {
            set_status(status, kStatusCapacity);
            n = uint32_t(cap);
        }
        counts[d] = int32_t(n);
    }
}

// CTAs stride over the received rows [world][cap]; per live row and local
// pair, w * down (rounded) goes to the source's block at (token, rank q).
// Then the tagged done flags to every rank.
__global__ void __launch_bounds__(256) ep_back_kernel(PrefillWork w, EpInbox in, int world, int rank, int per_rank,
                                                      int cap, EpPeers peers, uint32_t tag, unsigned *arrive) {
    const int rows = world * cap;
    for (int j = blockIdx.x; j < rows; j += gridDim.x) {
        const int s = j / cap;
        if (j - s * cap >= w.seg_count[s]) {
            continue;
        }
        const int t = in.src[j];
        if (t < 0 || t >= cap) {  // a row the source did not write this call
            set_status(w.status, kStatusBadShape);
            continue;
        }
        float *back = ep_inbox_at(peers.base[s], world, cap).back;
        for (int q = 0; q < kTopK; ++q) {
            const int e = in.idx[size_t(j) * 4 + q];
            if (e < 0 || owner_of(e, per_rank) != rank) {
                continue;
            }
            const int slot = w.pair_slot[size_t(j) * 4 + q];
            if (slot < 0) {
                continue;
            }
            const float wt = in.w[size_t(j) * 4 + q];
            const float4 *src = reinterpret_cast<const float4 *>(w.down + size_t(slot) * kDim);
            float4 *dst = reinterpret_cast<float4 *>(back + (size_t(t) * 4 + q) * kDim);
            for (int i = threadIdx.x; i < kDim / 4; i += blockDim.x) {
                const float4 v = src[i];
                dst[i] = make_float4(__fmul_rn(wt, v.x), __fmul_rn(wt, v.y), __fmul_rn(wt, v.z), __fmul_rn(wt, v.w));
            }
        }
    }
    publish_last(peers, world, cap, rank, true, arrive, [&](int) { return tagged_word(tag, 0u); });
}

// One CTA per own token: out = sum over its experts in ascending id of the
// returned rows w * down (src/model.cpp:450-459).
__global__ void ep_combine_kernel(const int32_t *__restrict__ idx, const float *__restrict__ back,
                                  float *__restrict__ out) {
    const int t = blockIdx.x;
    int e[4];
#pragma unroll
    for (int q = 0; q < kTopK; ++q) {
        e[q] = idx[size_t(t) * 4 + q];
    }
    int order[4] = {0, 1, 2, 3};  // ascending expert id (the four ids are distinct)
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
    const float *rows = back + size_t(t) * 4 * kDim;
    for (int c = threadIdx.x; c < kDim; c += blockDim.x) {
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < kTopK; ++i) {
            o = __fadd_rn(o, __ldcg(rows + size_t(order[i]) * kDim + c));
        }
        out[size_t(t) * kDim + c] = o;
    }
}

}  // namespace

// Largest shared-memory carveout for the dispatch kernels too (they run
// between the tensor-core kernels on the same stream).
void configure_prefill_ep() {
    cudaFuncSetAttribute(ep_plan_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    cudaFuncSetAttribute(ep_send_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    cudaFuncSetAttribute(ep_wait_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    cudaFuncSetAttribute(ep_back_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
    cudaFuncSetAttribute(ep_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
}

void launch_ep_plan(const int32_t *idx, int tokens, int world, int per_rank, int32_t *tok_off, int32_t *cnt,
                    cudaStream_t stream) {
    ep_plan_kernel<<<world, 1024, 0, stream>>>(idx, tokens, world, per_rank, tok_off, cnt);
}

void launch_ep_send(const float *x, const int32_t *idx, const float *wts, int tokens, int world, int rank, int cap,
                    const int32_t *tok_off, const int32_t *cnt, const EpPeers &peers, uint32_t tag,
                    unsigned *arrive, int sms, cudaStream_t stream) {
    ep_send_kernel<<<std::max(1, std::min(tokens, 2 * sms)), 256, 0, stream>>>(x, idx, wts, tokens, world, rank, cap,
                                                                               tok_off, cnt, peers, tag, arrive);
}

void launch_ep_wait(const unsigned long long *flags, int world, uint32_t tag, int cap, int32_t *counts,
                    uint32_t *status, cudaStream_t stream) {
    ep_wait_kernel<<<1, 32, 0, stream>>>(flags, world, tag, cap, counts, status);
}

void launch_ep_back(const PrefillWork &w, const EpInbox &in, int world, int rank, int per_rank, int cap,
                    const EpPeers &peers, uint32_t tag, unsigned *arrive, int sms, cudaStream_t stream) {
    ep_back_kernel<<<std::max(1, std::min(world * cap, 2 * sms)), 256, 0, stream>>>(w, in, world, rank, per_rank, cap,
                                                                                  peers, tag, arrive);
}

void launch_ep_combine(const int32_t *idx, int tokens, const float *back, float *out, cudaStream_t stream) {
    ep_combine_kernel<<<tokens, 256, 0, stream>>>(idx, back, out);
}

}  // namespace ttl
