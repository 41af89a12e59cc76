// decode_tc.cu -- persistent decode kernel on the tcgen05 tensor cores.
//
// Reference: GptOssModel::moe (tt-lab src/model.cpp:292-338) and the per-layer
// RMSNorm -> moe -> residual sequence of GptOssModel::forward
// (src/model.cpp:590-594).  One cooperative launch runs every token x layer of
// a decode call; one CTA per SM.
//
// Per layer:
//   A  select   Every CTA reads the layer's router sums (f64, accumulated by
//               the previous layer's epilogues -- the RMSNorm scale is a
//               scalar, so logit_e = b_e + s * sum_c W_ec g_c x_c splits over
//               row slices), picks the same top 4 and splits h = RMSNorm(x)*g
//               into four E4M3 terms (the B operand, N = 8).  Mode 0 (one
//               plain MoE, h given) computes the logits in a router phase with
//               an error bound instead and re-evaluates near-ties exactly in
//               the reference's order, so its indices equal the reference's.
//   B  gate/up  Units are (tile, K-block): a tile is 64 gate rows + the 64 up
//               rows of the same outputs of one selected expert (M = 128).
//               Each CTA takes an equal contiguous range of units (stream-K).
//               Loader warps copy the E2M1 nibbles straight from HBM into
//               shared memory (8-byte runs into 16-byte slots) and the block
//               scales into tensor memory; one thread issues block-scaled
//               MXF8F6F4 MMAs (K = 32) accumulating in tensor memory; epilogue
//               warps read the tile partial.  The last contributor to a tile
//               sums the partials in order, adds the biases, applies SwiGLU
//               and the routing weight, and writes the tile's 64 hidden values
//               as E4M3 terms -- the B operand of the down projection.
//   -- grid barrier --
//   C  down     Units are (128-row tile, expert x K-block): the four experts'
//               down projections accumulate into one tensor (the routing
//               weights are already in B).  The last contributor adds
//               sum_q w_q b_q, the residual, writes the output rows and (stack
//               mode) accumulates the next layer's router sums for them.
//   -- grid barrier --
// Every wait is bounded; on timeout the kernel records kStatusWaitTimeout,
// drains its own copies and MMAs, frees its tensor memory and returns.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace ttl {
namespace {

constexpr int kTerms = 4;
constexpr int kN = 8;
constexpr int kChunks = kDim / 16;            // 180 16-element K-chunks
constexpr int kSfChunks = (kBlocks + 3) / 4;  // 23 scale chunks of 4 K-blocks
constexpr int kStages = 9;
constexpr int kStageKB = 4;                   // K-blocks per stage
constexpr int kEpiWarps = 4;                  // warps 0-3
constexpr int kLoadWarps = 4;                 // warps 4-7
constexpr int kThreads = 32 * (kEpiWarps + kLoadWarps + 1);
constexpr int kGateTiles = kDim / 64;         // 45 tiles of 64 gate + 64 up rows
constexpr int kDownTiles = (kDim + 127) / 128;  // 23 tiles of 128 rows
constexpr int kMaxSlots = 16;                 // contributors per tile (checked)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD = 0;                                  // 2 x 8 columns
constexpr uint32_t kColSfa = 16;                               // kStages x 4 columns
constexpr uint32_t kColSfbG = kColSfa + 4 * kStages;           // 23 scale chunks x 4 columns
constexpr uint32_t kColSfbD = kColSfbG + 4 * ((kBlocks + 3) / 4);  // kDownSlots x 23 x 4 columns
constexpr int kDownSlots = 2;                 // down-projection experts a CTA touches (checked)
static_assert(kColSfbD + 4 * kDownSlots * ((kBlocks + 3) / 4) <= kTmemCols, "tensor memory map");
constexpr unsigned long long kSpinLimit = 1ull << 22;  // x ~0.6 us per poll: ~2.5 s

struct alignas(128) Smem {
    uint8_t a[kStages][16][2 * kStageKB][8][16];  // A stages: [row group][chunk][row][16 B]
    uint8_t sfa[kStages][32][4][4];               // A scales per stage: [m0][m1][K-block], rows m0 + 32*m1
    uint8_t bgu[kChunks][kN][16];                 // gate/up B: h terms
    uint8_t bdown[kDownSlots][kChunks][kN][16];   // down B: w * hidden terms of this CTA's experts
    uint8_t sfbg[kBlocks][kTerms];                // gate/up B term scales
    uint8_t sfbd[kDownSlots][kBlocks][kTerms];    // down B term scales
    int dslot[kTopK];                             // expert slot -> bdown slot, -1 if unused
    float xch[64];                                // up values for the SwiGLU exchange
    float part[128];                              // scratch for the tile reduction
    float logit[kMaxExperts];
    float bound[kMaxExperts];
    float val[kMaxExperts];
    double red[kThreads / 32];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t fin;
    uint32_t tmem;
    int go;      // grid-barrier verdict, written by thread 0 only
    int epi_go;  // epilogue verdict, written by thread 0 only
    int sel[kTopK];
    int local[kTopK];
    int slot_of[kTopK];
    float wts[kTopK];
    int n_local;
    int amb;
    int abort;
    int last;
    float scale;
};

// Role-local pipeline counters (each role walks the same unit sequence).
struct Pipe {
    uint32_t stage = 0;  // stages issued / consumed so far
    uint32_t seg = 0;    // segments (D buffers) so far
};

__device__ __forceinline__ bool aborted(const Smem &s) {
    return *reinterpret_cast<const volatile int *>(&s.abort) != 0;
}

__device__ __forceinline__ void fail_wait(Smem &s, uint32_t *status) {
    set_status(status, kStatusWaitTimeout);
    *reinterpret_cast<volatile int *>(&s.abort) = 1;
}

__device__ __forceinline__ bool wait_bar(Smem &s, uint64_t *bar, uint32_t parity, uint32_t *status) {
    if (aborted(s)) {
        return false;
    }
    if (!tc::mbar_wait(bar, parity)) {
        fail_wait(s, status);
        return false;
    }
    return true;
}

// Warp-uniform variants: lane 0 decides, the warp follows (warp-collective
// tcgen05 instructions need every lane).
__device__ __forceinline__ bool warp_aborted(const Smem &s) {
    return __shfl_sync(0xffffffffu, aborted(s) ? 1 : 0, 0) != 0;
}

__device__ __forceinline__ bool warp_wait(Smem &s, uint64_t *bar, uint32_t parity, uint32_t *status) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) {
        ok = wait_bar(s, bar, parity, status) ? 1 : 0;
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(tc::smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void epi_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Bounded grid barrier (all threads of every CTA).
__device__ bool grid_barrier(unsigned *bar, unsigned &gen, uint32_t *status, Smem &s) {
    __syncthreads();
    if (threadIdx.x == 0 && !aborted(s)) {
        __threadfence();
        const unsigned arrived = atomicAdd(&bar[0], 1u);
        if (arrived == gridDim.x - 1) {
            bar[0] = 0u;
            __threadfence();
            atomicExch(&bar[1], gen + 1u);
        } else {
            unsigned long long spins = 0;
            unsigned cur;
            while (true) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(bar + 1) : "memory");
                if (cur != gen) {
                    break;
                }
                if (++spins > kSpinLimit) {
                    fail_wait(s, status);
                    break;
                }
                __nanosleep(64);
            }
        }
        gen += 1u;
        __threadfence();
    }
    if (threadIdx.x == 0) {
        s.go = aborted(s) ? 0 : 1;
    }
    __syncthreads();
    return s.go != 0;
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Stage stamps for profiling (thread 0 of CTA 0; point 9 = latest phase-B end over CTAs).
__device__ __forceinline__ void stamp(const StackArgs &a, int step, int point) {
    if (a.trace && step < a.trace_steps && threadIdx.x == 0) {
        const unsigned long long t = globaltimer();
        if (blockIdx.x == 0) {
            a.trace[size_t(step) * kTracePoints + point] = t;
        }
        if (point == 3 || point == 6) {
            atomicMax(&a.trace[size_t(step) * kTracePoints + (point == 3 ? 8 : 9)], t);
        }
    }
}

// Contiguous unit range of CTA c out of g over `units` units.
__device__ __forceinline__ int range_lo(int c, int g, int units) {
    return int((long long)c * units / g);
}

__device__ __forceinline__ int cta_of(int u, int g, int units) {
    int c = int((long long)u * g / units);
    while (c + 1 < g && range_lo(c + 1, g, units) <= u) {
        ++c;
    }
    while (c > 0 && range_lo(c, g, units) > u) {
        --c;
    }
    return c;
}

// One GEMV phase: `tiles` tiles of `kunits` K-units each, stream-K over the grid.
struct Phase {
    int kind;    // 0 gate/up, 1 down
    int tiles;
    int kunits;  // K-units per tile (90 for gate/up, n_local * 90 for down)
};

struct Ctx {
    const StackArgs *a;
    const StackLayer *L;
    Smem *s;
    uint32_t tbase;
};

// Stages are aligned to scale chunks: K-blocks [4g, 4g+4) of one matrix (the
// last chunk of a row has 2), clipped to the segment.  Returns the stage's
// first K-unit offset within the tile and its K-block count.
__device__ __forceinline__ int stage_len(const Phase &p, int ku, int seg_left) {
    const int kb = ku % kBlocks;
    const int chunk_end = min((kb & ~3) + 4, kBlocks);
    return min(chunk_end - kb, seg_left);
}

// ---- loader warps (4-7) ----
// Thread lt copies chunk lt & 7 of rows (lt >> 3) + 16k, k = 0..7, of every
// stage, and the scale word of row lt.  Row addresses are formed once per
// segment (and per expert change in the down phase) and kept in registers.
__device__ void run_loader(const Ctx &c, const Phase &p, Pipe &pp) {
    Smem &s = *c.s;
    const int lt = threadIdx.x - 32 * kEpiWarps;  // 0..127
    const int ch = lt & 7;
    const int r_first = lt >> 3;
    const int units = p.tiles * p.kunits;
    const int u0 = range_lo(blockIdx.x, gridDim.x, units);
    const int u1 = range_lo(blockIdx.x + 1, gridDim.x, units);
    const uint8_t *gate = c.L->gate;
    const uint8_t *up = c.L->up;
    const uint8_t *down = c.L->down;
    int u = u0;
    while (u < u1) {
        const int tile = u / p.kunits;
        const int seg_end = min(u1, (tile + 1) * p.kunits);
        int cur_q = -1;
        const uint8_t *rowp[8];   // nibble rows of this thread (nullptr past the matrix)
        const uint8_t *sfrow = nullptr;
        while (u < seg_end) {
            if (warp_aborted(s)) {
                return;
            }
            const int ku0 = u - tile * p.kunits;
            const int q = ku0 / kBlocks;
            if (q != cur_q) {
                cur_q = q;
                if (p.kind == 0) {
                    const int qq = tile / kGateTiles;
                    const int j = tile - qq * kGateTiles;
                    const size_t off = size_t(s.local[s.slot_of[qq]]) * kPackedMatrixBytes;
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int i = r_first + 16 * k;
                        rowp[k] = (i < 64 ? gate : up) + off + size_t(64 * j + (i & 63)) * kNibbleRowBytes;
                    }
                    sfrow = (lt < 64 ? gate : up) + off + kNibbleBytes + size_t(64 * j + (lt & 63)) * kScaleRowBytes;
                } else {
                    const uint8_t *m = down + size_t(s.local[s.slot_of[q]]) * kPackedMatrixBytes;
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int row = 128 * tile + r_first + 16 * k;
                        rowp[k] = row < kDim ? m + size_t(row) * kNibbleRowBytes : nullptr;
                    }
                    const int row = 128 * tile + lt;
                    sfrow = row < kDim ? m + kNibbleBytes + size_t(row) * kScaleRowBytes : nullptr;
                }
            }
            const int nkb = stage_len(p, ku0, seg_end - u);
            const int kb0 = ku0 % kBlocks;
            const uint32_t st = pp.stage % kStages;
            const uint32_t use = pp.stage / kStages;
            if (use > 0 && !warp_wait(s, &s.empty[st], (use - 1) & 1, c.a->status)) {
                return;
            }
            const int j = (ch >> 1) - (kb0 & 3);  // K-block of the stage this thread's chunk belongs to
            if (j >= 0 && j < nkb) {
                const size_t koff = size_t(kb0 + j) * 16 + (ch & 1) * 8;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (rowp[k]) {
                        const int i = r_first + 16 * k;
                        cp_async8(&s.a[st][i >> 3][ch][i & 7][0], rowp[k] + koff);
                    }
                }
            }
            if (sfrow) {
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(tc::smem_u32(&s.sfa[st][lt & 31][lt >> 5][0])),
                             "l"(sfrow + (kb0 & ~3))
                             : "memory");
            }
            cp_async_arrive(&s.full[st]);
            ++pp.stage;
            u += nkb;
        }
    }
}

// L2 prefetch (idle lanes of the MMA warp during gate/up): this CTA's
// down-phase rows, so the down phase streams from L2.
__device__ void prefetch_down(const Ctx &c, int kunits) {
    const Smem &s = *c.s;
    const int lane = threadIdx.x & 31;
    const int units = kDownTiles * kunits;
    const int u0 = range_lo(blockIdx.x, gridDim.x, units);
    const int u1 = range_lo(blockIdx.x + 1, gridDim.x, units);
    for (int u = u0; u < u1;) {
        const int tile = u / kunits;
        const int ku = u - tile * kunits;
        const int q = ku / kBlocks;
        const int kb0 = ku % kBlocks;
        const int kb1 = min(kBlocks, kb0 + (u1 - u));
        const uint8_t *m = c.L->down + size_t(s.local[s.slot_of[q]]) * kPackedMatrixBytes;
        for (int i = lane - 1; i < 128; i += 31) {
            const int row = 128 * tile + i;
            if (row < kDim) {
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(m + size_t(row) * kNibbleRowBytes + kb0 * 16),
                             "r"(uint32_t((kb1 - kb0) * 16))
                             : "memory");
            }
        }
        u += kb1 - kb0;
    }
}

// ---- MMA issuer (warp 8, lane 0) ----
__device__ void run_mma(const Ctx &c, const Phase &p, Pipe &pp) {
    Smem &s = *c.s;
    const int units = p.tiles * p.kunits;
    const int u0 = range_lo(blockIdx.x, gridDim.x, units);
    const int u1 = range_lo(blockIdx.x + 1, gridDim.x, units);
    const uint32_t a0 = tc::smem_u32(&s.a[0][0][0][0][0]);
    const uint32_t idesc0 = tc::instr_desc(kN, 0, 0);
    int u = u0;
    while (u < u1 && !aborted(s)) {
        const int tile = u / p.kunits;
        const int seg_end = min(u1, (tile + 1) * p.kunits);
        const uint32_t db = pp.seg & 1;
        const uint32_t duse = pp.seg >> 1;
        if (duse > 0 && !wait_bar(s, &s.acc_empty[db], (duse - 1) & 1, c.a->status)) {
            return;
        }
        tc::fence_after_sync();
        bool first = true;
        while (u < seg_end && !aborted(s)) {
            const int ku0 = u - tile * p.kunits;
            const int nkb = stage_len(p, ku0, seg_end - u);
            const uint32_t st = pp.stage % kStages;
            const uint32_t use = pp.stage / kStages;
            if (!wait_bar(s, &s.full[st], use & 1, c.a->status)) {
                return;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc::fence_after_sync();
            tc::sf_copy(c.tbase + kColSfa + 4 * st, tc::smem_u32(&s.sfa[st][0][0][0]));
            for (int j = 0; j < nkb; ++j) {
                const int ku = ku0 + j;
                const int kb = ku % kBlocks;
                uint32_t bbase, sfb;
                if (p.kind == 0) {
                    bbase = tc::smem_u32(&s.bgu[0][0][0]);
                    sfb = c.tbase + kColSfbG + 4 * (kb >> 2);
                } else {
                    const int ds = s.dslot[ku / kBlocks];
                    bbase = tc::smem_u32(&s.bdown[ds][0][0][0]);
                    sfb = c.tbase + kColSfbD + 4 * (ds * kSfChunks + (kb >> 2));
                }
                const uint64_t ad =
                    tc::smem_desc(a0 + st * sizeof(s.a[0]) + uint32_t(kb & 3) * 256, 128, 2 * kStageKB * 128);
                const uint64_t bd = tc::smem_desc(bbase + uint32_t(kb) * 256, 128, kChunks * 128);
                const uint32_t idesc = idesc0 | (uint32_t(kb & 3) << 4) | (uint32_t(kb & 3) << 29);
                tc::mma(c.tbase + kColD + 8 * db, ad, bd, idesc, (c.tbase + kColSfa + 4 * st) | (uint32_t(kb & 3) << 30),
                        sfb | (uint32_t(kb & 3) << 30), !first);
                first = false;
            }
            tc::mma_commit(&s.empty[st]);
            ++pp.stage;
            u += nkb;
        }
        tc::mma_commit(&s.acc_full[db]);
        ++pp.seg;
    }
}

// Number of contributors to tile t and the slot of this CTA.
__device__ __forceinline__ void tile_slots(const Phase &p, int tile, int &n, int &slot) {
    const int units = p.tiles * p.kunits;
    const int c0 = cta_of(tile * p.kunits, gridDim.x, units);
    const int c1 = cta_of((tile + 1) * p.kunits - 1, gridDim.x, units);
    n = c1 - c0 + 1;
    slot = int(blockIdx.x) - c0;
}

// ---- epilogue warps (0-3): one thread per tile row ----
__device__ void run_epilogue(const Ctx &c, const Phase &p, Pipe &pp, int t_token, int li, bool next_router) {
    Smem &s = *c.s;
    const StackArgs &a = *c.a;
    const StackLayer &L = *c.L;
    const int i = threadIdx.x;  // 0..127: tile row
    const int w = i >> 5;
    const int lane = i & 31;
    const int units = p.tiles * p.kunits;
    const int u0 = range_lo(blockIdx.x, gridDim.x, units);
    const int u1 = range_lo(blockIdx.x + 1, gridDim.x, units);
    int u = u0;
    while (u < u1) {
        const int tile = u / p.kunits;
        const int seg_end = min(u1, (tile + 1) * p.kunits);
        const uint32_t db = pp.seg & 1;
        const uint32_t duse = pp.seg >> 1;
        if (i == 0) {
            s.epi_go = wait_bar(s, &s.acc_full[db], duse & 1, a.status) ? 1 : 0;
        }
        epi_sync();  // s.epi_go is the same for all epilogue threads
        const bool go = s.epi_go != 0;
        epi_sync();  // nobody rewrites s.epi_go before everyone has read it
        if (!go) {
            return;
        }
        tc::fence_after_sync();
        float d[8];
        tc::tmem_ld8(c.tbase + (uint32_t(32 * w) << 16) + kColD + 8 * db, d);
        tc::wait_ld();
        tc::fence_before_sync();
        mbar_arrive(&s.acc_empty[db]);
        ++pp.seg;
        u = seg_end;
        float part = 0.0f;
#pragma unroll
        for (int n = 0; n < kTerms; ++n) {
            part += d[n];
        }
        int nslot, slot;
        tile_slots(p, tile, nslot, slot);
        if (nslot > kMaxSlots) {
            if (i == 0) {
                set_status(a.status, kStatusBadShape);
            }
            continue;
        }
        float *ws = (p.kind == 0 ? a.part_gu : a.part_dn) + (size_t(tile) * kMaxSlots + slot) * 128;
        unsigned *cnt = (p.kind == 0 ? a.cnt_gu : a.cnt_dn) + tile;
        if (nslot > 1) {
            ws[i] = part;
            __threadfence();
            epi_sync();
            if (i == 0) {
                const unsigned prev = atomicAdd(cnt, 1u);
                s.last = (prev == unsigned(nslot - 1));
                if (s.last) {
                    *cnt = 0u;
                }
            }
            epi_sync();
            if (!s.last) {
                continue;
            }
            __threadfence();
            float sum = 0.0f;
            const float *base = (p.kind == 0 ? a.part_gu : a.part_dn) + size_t(tile) * kMaxSlots * 128;
            for (int k = 0; k < nslot; ++k) {
                sum += (k == slot) ? part : __ldcg(base + k * 128 + i);
            }
            part = sum;
        }
        if (p.kind == 0) {
            // gate rows 0..63 (warps 0, 1), up rows 64..127 (warps 2, 3)
            const int q = tile / kGateTiles;
            const int j = tile - q * kGateTiles;
            const int le = s.local[s.slot_of[q]];
            const int row = 64 * j + (i & 63);
            if (i >= 64) {
                s.xch[i - 64] = __fadd_rn(L.up_b[size_t(le) * kDim + row], part);
            }
            epi_sync();
            if (i < 64) {
                const float g = __fadd_rn(L.gate_b[size_t(le) * kDim + row], part);
                const float h = __fmul_rn(swiglu_ref(g, s.xch[i]), s.wts[s.slot_of[q]]);
                uint32_t sc;
                const uint32_t tb = tc::split_terms<kTerms>(h, sc);
                const int k = row;  // down-projection K index
                uint8_t *bd = a.bdown + (size_t(q) * kChunks + (k >> 4)) * kN * 16;
#pragma unroll
                for (int n = 0; n < kTerms; ++n) {
                    bd[n * 16 + (k & 15)] = uint8_t(tb >> (8 * n));
                }
                if (lane == 0) {
                    const int kb = k >> 5;
#pragma unroll
                    for (int n = 0; n < kTerms; ++n) {
                        a.sfb_down[(size_t(q) * kBlocks + kb) * kTerms + n] = uint8_t(sc >> (8 * n));
                    }
                }
            }
            epi_sync();
        } else {
            const int row = 128 * tile + i;
            if (row < kDim) {
                float bsum = 0.0f;
                for (int k = 0; k < s.n_local; ++k) {
                    const int rank = s.slot_of[k];
                    bsum = __fadd_rn(bsum, __fmul_rn(s.wts[rank], L.down_b[size_t(s.local[rank]) * kDim + row]));
                }
                const float o = __fadd_rn(part, bsum);
                const float *xcur = (li == 0) ? a.x + size_t(t_token) * kDim : a.y + size_t(t_token) * kDim;
                float *ycur = a.y + size_t(t_token) * kDim;
                const float yv = (a.mode == 1) ? __fadd_rn(__ldcg(xcur + row), o) : o;
                ycur[row] = yv;
                s.part[i] = yv;
            }
            if (next_router) {
                // router sums of the next (token, layer) over these rows
                epi_sync();
                const bool more_layers = (li + 1 < a.layer_end - a.layer_begin);
                const StackLayer &N = a.layers[more_layers ? a.layer_begin + li + 1 : a.layer_begin];
                const int step = t_token * (a.layer_end - a.layer_begin) + li;
                double *acc = a.acc + size_t((step + 1) & 1) * (kMaxExperts + 1);
                for (int e = w; e < a.experts + 1; e += kEpiWarps) {
                    double v = 0.0;
#pragma unroll
                    for (int r4 = 0; r4 < 4; ++r4) {
                        const int rr = lane + 32 * r4;
                        const int r = 128 * tile + rr;
                        if (r < kDim) {
                            const float xr = more_layers ? s.part[rr] : __ldcg(a.x + size_t(t_token + 1) * kDim + r);
                            v += (e < a.experts)
                                     ? double(__ldg(N.router_w + size_t(e) * kDim + r)) * double(__fmul_rn(xr, N.norm_w[r]))
                                     : double(__fmul_rn(xr, xr));
                        }
                    }
                    v = warp_sum_d(v);
                    if (lane == 0) {
                        atomicAdd(acc + e, v);
                    }
                }
            }
        }
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

__device__ float exact_logit(const float *__restrict__ wrow, float bias, const float *__restrict__ h) {
    float acc = bias;
    for (int c = 0; c < kDim; c += 8) {
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            p[j] = __fmul_rn(__ldg(wrow + c + j), __ldcg(h + c + j));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            acc = __fadd_rn(acc, p[j]);
        }
    }
    return acc;
}

// Warp 0: top 4 of s.logit (lowest index on exact ties); with bounds, flags
// an interval of a selected expert touching another expert's.
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

__global__ void __launch_bounds__(kThreads, 1) decode_tc_kernel(StackArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem &s = *reinterpret_cast<Smem *>(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int E = a.experts;
    const int nl = a.layer_end - a.layer_begin;
    unsigned gen = 0;

    if (threadIdx.x == 0) {
        s.abort = 0;
        gen = *reinterpret_cast<volatile unsigned *>(a.barrier + 1);
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&s.full[i], 32 * kLoadWarps);
            tc::mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.acc_full[i], 1);
            tc::mbar_init(&s.acc_empty[i], 32 * kEpiWarps);
        }
        tc::mbar_init(&s.fin, 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&s.tmem, kTmemCols);
        tc::tmem_relinquish();
    }
    // zero the unused B rows (terms 4..7) once
    for (int i = threadIdx.x; i < kChunks * kN * 16 / 16; i += kThreads) {
        const int ch = i / kN, n = i % kN;
        if (n >= kTerms) {
            *reinterpret_cast<uint4 *>(&s.bgu[ch][n][0]) = make_uint4(0, 0, 0, 0);
            for (int q = 0; q < kDownSlots; ++q) {
                *reinterpret_cast<uint4 *>(&s.bdown[q][ch][n][0]) = make_uint4(0, 0, 0, 0);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = s.tmem;
    Pipe pipe;

    // Router sums of (token 0, first layer) in stack mode.
    if (a.mode == 1) {
        const StackLayer &L = a.layers[a.layer_begin];
        const int r0 = range_lo(blockIdx.x, gridDim.x, kDim);
        const int r1 = range_lo(blockIdx.x + 1, gridDim.x, kDim);
        for (int e = warp; e < E + 1; e += kThreads / 32) {
            const int r = r0 + lane;
            double v = 0.0;
            if (r < r1) {
                const float xr = a.x[r];
                v = (e < E) ? double(__ldg(L.router_w + size_t(e) * kDim + r)) * double(__fmul_rn(xr, L.norm_w[r]))
                            : double(__fmul_rn(xr, xr));
            }
            v = warp_sum_d(v);
            if (lane == 0) {
                atomicAdd(a.acc + e, v);
            }
        }
    }
    bool ok = grid_barrier(a.barrier, gen, a.status, s);

    for (int t = 0; ok && t < a.tokens; ++t) {
        for (int li = 0; ok && li < nl; ++li) {
            const int l = a.layer_begin + li;
            const StackLayer &L = a.layers[l];
            const int step = t * nl + li;
            const float *xcur = (li == 0) ? a.x + size_t(t) * kDim : a.y + size_t(t) * kDim;

            stamp(a, step, 0);
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
                if (blockIdx.x == 0) {
                    double *other = a.acc + size_t((step + 1) & 1) * (kMaxExperts + 1);
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
                // CTA e < E: expert e's logit and the bound on the reference's f32 chain.
                for (int e = blockIdx.x; e < E; e += gridDim.x) {
                    const float *wr = L.router_w + size_t(e) * kDim;
                    constexpr int kCols = kDim / (kThreads / 32);  // 320 per warp
                    constexpr int kPer = (kCols + 31) / 32;        // 10 per lane
                    const int c0 = warp * kCols;
                    float p[kPer];
                    double loc = 0.0;
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        const int off = lane * kPer + j;
                        p[j] = (off < kCols) ? __fmul_rn(__ldg(wr + c0 + off), __ldcg(xcur + c0 + off)) : 0.0f;
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
                    double total = 0.0;
                    for (int k = 0; k < kThreads / 32; ++k) {
                        if (k < warp) {
                            base += s.red[k];
                        }
                        total += s.red[k];
                    }
                    double run = base + inc - loc;
                    double abs_sum = 0.0;
#pragma unroll
                    for (int j = 0; j < kPer; ++j) {
                        run += double(p[j]);
                        abs_sum += fabs(run);
                    }
                    abs_sum = warp_sum_d(abs_sum);
                    __syncthreads();
                    if (lane == 0) {
                        s.red[warp] = abs_sum;
                    }
                    __syncthreads();
                    if (threadIdx.x == 0) {
                        double abs_total = 0.0;
                        for (int k = 0; k < kThreads / 32; ++k) {
                            abs_total += s.red[k];
                        }
                        const double logit = double(L.router_b[e]) + total;
                        a.logits[e] = float(logit);
                        a.bounds[e] = float((1.02 * 5.9604644775390625e-08 * abs_total +
                                             5.9604644775390625e-08 * fabs(logit) + 1e-30) * 1.0001);
                    }
                    __syncthreads();
                }
                ok = grid_barrier(a.barrier, gen, a.status, s);
                if (!ok) {
                    break;
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
                            s.val[e] = exact_logit(L.router_w + size_t(e) * kDim, L.router_b[e], xcur);
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
            stamp(a, step, 1);
            // softmax (src/model.cpp:310-321) and ownership
            if (threadIdx.x == 0) {
                float maximum = -INFINITY;
                float v[4], wv[4];
                for (int q = 0; q < kTopK; ++q) {
                    v[q] = s.val[s.sel[q]];
                    maximum = (maximum < v[q]) ? v[q] : maximum;
                }
                float sum = 0.0f;
                for (int q = 0; q < kTopK; ++q) {
                    wv[q] = expf(__fsub_rn(v[q], maximum));
                    sum = __fadd_rn(sum, wv[q]);
                }
                int n = 0;
                for (int q = 0; q < kTopK; ++q) {
                    s.wts[q] = __fdiv_rn(wv[q], sum);
                    const int le = s.sel[q] - a.expert_begin;
                    s.local[q] = (le >= 0 && le < a.expert_count) ? le : -1;
                    if (s.local[q] >= 0) {
                        s.slot_of[n++] = q;
                    }
                }
                s.n_local = n;
                if (blockIdx.x == 0 && t == a.tokens - 1 && li == nl - 1) {
                    for (int q = 0; q < kTopK; ++q) {
                        a.top_idx[q] = s.sel[q];
                        a.top_w[q] = s.wts[q];
                    }
                }
            }
            __syncthreads();
            // B for gate/up: h split into terms; SFB into tensor memory.
            // this warp's K-blocks: kb2 = warp + 9 i, 5 passes of two blocks;
            // all x (and norm weight) loads are issued up front
            constexpr int kPasses = (kBlocks / 2 + kThreads / 32 - 1) / (kThreads / 32);
            float xr[kPasses][2], gr[kPasses][2];
#pragma unroll
            for (int pi = 0; pi < kPasses; ++pi) {
                const int kb2 = warp + pi * (kThreads / 32);
#pragma unroll
                for (int z = 0; z < 2; ++z) {
                    const int k = (2 * kb2 + z) * 32 + lane;
                    xr[pi][z] = kb2 < kBlocks / 2 ? __ldcg(xcur + k) : 0.0f;
                    gr[pi][z] = (kb2 < kBlocks / 2 && a.mode == 1) ? __ldg(L.norm_w + k) : 1.0f;
                }
            }
#pragma unroll
            for (int pi = 0; pi < kPasses; ++pi) {
                const int kb2 = warp + pi * (kThreads / 32);
                if (kb2 >= kBlocks / 2) {
                    break;
                }
                // two independent K-blocks per pass (interleaved dependency chains)
                float h[2];
#pragma unroll
                for (int z = 0; z < 2; ++z) {
                    h[z] = (a.mode == 1) ? __fmul_rn(__fmul_rn(xr[pi][z], s.scale), gr[pi][z]) : xr[pi][z];
                }
                uint32_t sc[2], tb[2];
#pragma unroll
                for (int z = 0; z < 2; ++z) {
                    tb[z] = tc::split_terms<kTerms>(h[z], sc[z]);
                }
#pragma unroll
                for (int z = 0; z < 2; ++z) {
                    const int kb = 2 * kb2 + z;
                    const int k = kb * 32 + lane;
#pragma unroll
                    for (int n = 0; n < kTerms; ++n) {
                        s.bgu[k >> 4][n][k & 15] = uint8_t(tb[z] >> (8 * n));
                    }
                    if (lane == 0) {
#pragma unroll
                        for (int n = 0; n < kTerms; ++n) {
                            s.sfbg[kb][n] = uint8_t(sc[z] >> (8 * n));
                        }
                    }
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __threadfence_block();
            __syncthreads();
            if (warp >= kEpiWarps && warp < kEpiWarps + kLoadWarps) {
                const int q4 = warp & 3;
                for (int g = 0; g < kSfChunks; ++g) {
                    uint32_t v = 0;
                    if (lane < kTerms) {
                        for (int k = 0; k < 4; ++k) {
                            const int kb = 4 * g + k;
                            v |= (kb < kBlocks ? uint32_t(s.sfbg[kb][lane]) : 127u) << (8 * k);
                        }
                    }
                    tc::tmem_st4(tbase + (uint32_t(32 * q4) << 16) + kColSfbG + 4 * g, v, 0u, 0u, 0u);
                }
                tc::wait_st();
            }
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();

            stamp(a, step, 2);
            // ---------------- B: gate/up ----------------
            Ctx cx{&a, &L, &s, tbase};
            const Phase pb{0, s.n_local * kGateTiles, kBlocks};
            if (warp < kEpiWarps) {
                run_epilogue(cx, pb, pipe, t, li, false);
            } else if (warp < kEpiWarps + kLoadWarps) {
                run_loader(cx, pb, pipe);
            } else if (lane == 0) {
                run_mma(cx, pb, pipe);
            } else {
                prefetch_down(cx, s.n_local * kBlocks);
            }
            __syncthreads();
            stamp(a, step, 3);
            ok = grid_barrier(a.barrier, gen, a.status, s);
            if (!ok) {
                break;
            }
            stamp(a, step, 4);
            // ---------------- C: down ----------------
            // B for down: the w * hidden terms (written by phase B's reducers)
            // of the experts this CTA's down units touch (at most kDownSlots),
            // into shared memory; their scales into tensor memory.
            if (threadIdx.x == 0) {
                const int ku_tile = s.n_local * kBlocks;
                const int units = kDownTiles * ku_tile;
                const int u0 = range_lo(blockIdx.x, gridDim.x, units);
                const int u1 = range_lo(blockIdx.x + 1, gridDim.x, units);
                for (int q = 0; q < kTopK; ++q) {
                    s.dslot[q] = -1;
                }
                int nd = 0;
                for (int u = u0; u < u1;) {
                    const int ku = u % ku_tile;
                    const int q = ku / kBlocks;
                    if (s.dslot[q] < 0) {
                        if (nd < kDownSlots) {
                            s.dslot[q] = nd++;
                        } else {
                            set_status(a.status, kStatusBadShape);
                            s.dslot[q] = 0;
                        }
                    }
                    u += min(kBlocks - ku % kBlocks, u1 - u);
                }
            }
            __syncthreads();
            {
                constexpr int kPer = (kDownSlots * kChunks * kTerms + kThreads - 1) / kThreads;
                uint4 buf[kPer];
                int dst[kPer];
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    const int i = threadIdx.x + k * kThreads;  // over (q in 0..3, chunk, term) of used experts
                    dst[k] = -1;
                    int seen = 0;
                    for (int q = 0; q < kTopK; ++q) {
                        if (s.dslot[q] >= 0 && q < s.n_local) {
                            const int base = seen * kChunks * kTerms;
                            if (i >= base && i < base + kChunks * kTerms) {
                                const int r = i - base;
                                const int ch = r / kTerms;
                                const int n = r - ch * kTerms;
                                buf[k] = __ldcg(reinterpret_cast<const uint4 *>(a.bdown + ((size_t(q) * kChunks + ch) * kN + n) * 16));
                                dst[k] = (s.dslot[q] * kChunks + ch) * kN + n;
                            }
                            ++seen;
                        }
                    }
                }
#pragma unroll
                for (int k = 0; k < kPer; ++k) {
                    if (dst[k] >= 0) {
                        *reinterpret_cast<uint4 *>(&s.bdown[0][0][0][0] + size_t(dst[k]) * 16) = buf[k];
                    }
                }
            }
            for (int i = threadIdx.x; i < kTopK * kBlocks; i += kThreads) {
                const int q = i / kBlocks;
                if (q < s.n_local && s.dslot[q] >= 0) {
                    const uint32_t w4 = __ldcg(reinterpret_cast<const unsigned int *>(a.sfb_down) + i);
                    *reinterpret_cast<uint32_t *>(&s.sfbd[s.dslot[q]][i % kBlocks][0]) = w4;
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
            if (warp >= kEpiWarps && warp < kEpiWarps + kLoadWarps) {
                const int q4 = warp & 3;
                for (int d = 0; d < kDownSlots; ++d) {
                    for (int g = 0; g < kSfChunks; ++g) {
                        uint32_t v = 0;
                        if (lane < kTerms) {
                            for (int k = 0; k < 4; ++k) {
                                const int kb = 4 * g + k;
                                v |= (kb < kBlocks ? uint32_t(s.sfbd[d][kb][lane]) : 127u) << (8 * k);
                            }
                        }
                        tc::tmem_st4(tbase + (uint32_t(32 * q4) << 16) + kColSfbD + 4 * (d * kSfChunks + g), v, 0u, 0u,
                                     0u);
                    }
                }
                tc::wait_st();
            }
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            stamp(a, step, 5);
            const bool next_router =
                (a.mode == 1) && (li + 1 < nl || t + 1 < a.tokens);
            const Phase pc{1, kDownTiles, s.n_local * kBlocks};
            if (warp < kEpiWarps) {
                run_epilogue(cx, pc, pipe, t, li, next_router);
            } else if (warp < kEpiWarps + kLoadWarps) {
                run_loader(cx, pc, pipe);
            } else if (lane == 0) {
                run_mma(cx, pc, pipe);
            }
            __syncthreads();
            stamp(a, step, 6);
            ok = grid_barrier(a.barrier, gen, a.status, s);
            stamp(a, step, 7);
        }
    }
    // drain: this thread's copies; the MMA thread waits for its MMAs; then
    // tensor memory is freed
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (warp == kEpiWarps + kLoadWarps && lane == 0) {
        tc::mma_commit(&s.fin);
        tc::mbar_wait(&s.fin, 0);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
}

} // namespace

size_t decode_tc_smem_bytes() {
    return sizeof(Smem);
}

void configure_decode_tc() {
    cudaFuncSetAttribute(decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(Smem)));
}

cudaError_t launch_decode_tc(const StackArgs &args, int sms, cudaStream_t stream) {
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
    return cudaLaunchKernelEx(&cfg, decode_tc_kernel, args);
}

} // namespace ttl
