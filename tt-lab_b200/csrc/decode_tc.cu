// decode_tc.cu -- persistent decode kernel on the tcgen05 tensor cores.
//
// Reference: GptOssModel::moe (tt-lab src/model.cpp:292-338) and the per-layer
// RMSNorm -> moe -> residual sequence of GptOssModel::forward
// (src/model.cpp:590-594).  One cooperative launch runs every token x layer of
// a decode call; one CTA per SM.
//
// Roles (10 warps):
//   warps 0-8  the compute group: selection and B-operand preparation;
//              warps 0-3 also run the epilogues (one thread
//              per tile row, TMEM lane quadrant = warp); lane 0 of each of
//              warps 4-7 issues the block-scaled MMAs of one scale chunk of
//              every stage into its own accumulator (one issuing thread
//              sustains about one MMA per 150 cycles, four about one per 40);
//              lane 0 of warp 8 waits for and copies the down operand
//   warp 9     lane 0 issues the loads into the stage ring: per stage 32 KB
//              of packed E2M1 weights as two 128-byte x 128-row TMA boxes
//              (128-byte swizzle: the K-major layout of the MMA's A operand)
//              and their scales as bulk copies of the packed layout's 512-byte
//              tile blocks (already in tcgen05.cp order).  It follows the
//              published selection only, so the down-projection weights stream
//              in while the grid is still finishing the gate/up phase.
// Each CTA builds its work plans (stages and segments of both phases for 0..4
// local experts) once per launch; the roles walk them.
//
// Products are kind::mxf4 block-scaled MMAs (A = the weights' E2M1 nibbles
// with their E8M0 scales, untouched; K = 64 per instruction).  The B operand
// is the activation in block fixed point: 12 base-4 digit terms per value
// (E2M1 values 0..3 with a power-of-two scale per term and K-block, N = 16),
// exact to 2^-24 of each K-block's largest value; the accumulator's 16
// columns are the per-term partial products, summed in the epilogue.
//
// Per step (token x layer), with no grid barrier:
//   A  select   Every CTA polls the router sums the previous step's 23 down
//               tiles published as tagged words (each f64 sum as a hi / lo
//               pair in one 16-byte word pair), adds them in tile order (so
//               all CTAs get the same sums -- the RMSNorm scale is a scalar, so
//               logit_e = b_e + s * sum_c W_ec g_c x_c splits over row slices)
//               and picks the same top 4 (four rounds of warp max / min
//               reductions over order keys); then it loads the B operand those
//               tiles wrote (digit terms of x*g, counted separately: it is off
//               the critical path, behind the first weight loads).  The first
//               step of a launch splits h = RMSNorm(x)*g itself.
//               Mode 0 (one plain MoE, h given) computes the logits in a
//               router phase with an error bound instead (CTA e publishes
//               expert e's logit and bound as a tagged 16-byte pair that every
//               CTA polls) and re-evaluates near-ties exactly in the
//               reference's order, so its indices equal the reference's.
//   B  gate/up  Units are (tile, K-block pair): a tile is 128 gate rows and the 128
//               up rows of the same outputs of one selected expert (two M = 128
//               accumulators).  Each CTA takes an equal contiguous range of
//               units (stream-K).  The last contributor to a tile sums the
//               partials in order, adds the biases, applies SwiGLU and the
//               routing weight, writes the tile's 128 hidden values as digit
//               terms -- the B operand of the down projection -- and counts
//               the tile on its expert slot.
//   C  down     Units are (128-row tile, expert x K-block pair): the four experts'
//               down projections accumulate into one tensor (the routing
//               weights are already in B).  A CTA starts once the gate/up tiles
//               of the expert slots it reads are all counted.  The last
//               contributor adds sum_q w_q b_q, the residual, publishes the
//               next step's router sums over its rows (tagged words), then
//               writes the output rows and the next step's B operand and
//               counts the tile.
// Split-K partials and router sums travel as tagged words (value + step tag
// in one 8-byte store), so the reader polls the data itself -- no fence on
// the writer's side, and every poll round keeps all of a thread's missing
// words in flight together (poll_tagged); the tag base lives on the
// device and advances per launch, so a replayed graph never matches an old
// word.  Buffers alternate between even and odd steps: a CTA starts step
// s + 2 only after every CTA has contributed to step s + 1, so nothing of
// step s is still being read.
//
// Expert parallelism (world > 1): each rank runs this kernel over its own
// experts; the down reducers exchange the ranks' partial output rows as
// tagged words stored into each other's buffers over NVLink and add them in
// rank order (exchange_row), so every rank continues with the same bits.
// With more than 32 experts (decode_tc_kernel<true>) the down reducers stage
// the next layer's router weights of their rows in the idle stage ring (one
// 2-D tensor copy per tile, kTmaRouter).
// Every wait is bounded; on timeout the kernel records kStatusWaitTimeout,
// drains its own copies and MMAs, frees its tensor memory and returns.
#include <cuda_runtime.h>

#include <cstddef>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace ttl {
namespace {

constexpr int kN = 16;                        // B rows: tc::kDigitTerms digit terms + 4 zero rows
constexpr int kPairs = kBlocks / 2;           // 45 K-block pairs (one MMA each) per row
constexpr int kBRowBytes = 256;               // B bytes per K-block: [2 row groups][8 rows][16 B]
constexpr int kCodeBytes = 96;                // block codes per B operand (90 + padding, 127)
constexpr int kTiles = kScaleTiles;           // 23 tiles of 128 rows
constexpr int kStages = 4;
constexpr int kEpiWarps = 4;                  // warps 0-3
constexpr int kIssuers = 4;                   // MMA issuers: lane 0 of warps 4-7
constexpr int kIssuerWarp0 = 4;
constexpr int kMmaWarp = 8;                   // lane 0 issues the operand bulk copies
constexpr int kTmaWarp = 9;
constexpr int kThreads = 32 * (kTmaWarp + 1);
constexpr int kComputeWarps = kTmaWarp;       // warps 0-8
constexpr int kComputeThreads = 32 * kComputeWarps;
constexpr int kMaxSlots = 16;                 // contributors per tile (checked)
constexpr uint32_t kBoxTx = 128 * 128;        // bytes of one weight box (8 K-blocks of 128 rows)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD = 0;                                  // 2 buffers x kIssuers x 16 columns
constexpr uint32_t kColSfa = 128;                              // kStages x 4 chunks x 4 columns
constexpr uint32_t kSfbCols = 4 * 24;                          // B scales: 4 columns per chunk (the MMA's scale
                                                               // address is 4-column aligned), 23 chunks + 1
constexpr uint32_t kColSfbG = kColSfa + 16 * kStages;          // gate/up B scales
constexpr uint32_t kColSfbD = kColSfbG + kSfbCols;             // kDownSlots x kSfbCols
constexpr int kDownSlots = 2;                 // down-projection experts a CTA touches (checked)
static_assert(kColSfbD + kSfbCols * kDownSlots <= kTmemCols, "tensor memory map");
constexpr int kPreE = 32;                     // next-layer router weights the down epilogue loads early
static_assert(kPreE == kRouterMapFirstExpert, "the router tensor map's box starts past the preloaded experts");
constexpr int kOwnMax = 3;                    // tiles a CTA reduces in one phase (checked)
constexpr unsigned long long kGridWaitNs = 2000000000ull;

// ---- per-CTA work plans ----
// The stages and segments of one phase for one number of local experts,
// walked in the order every role uses (computed once per launch, so the
// per-stage loops do no unit arithmetic).
constexpr int kPlanStages = 24;  // stages of one phase (checked)
constexpr int kPlanSegs = 6;     // segments of one phase (checked)
struct PlanStage {
    uint8_t tile;   // 128-row tile of the expert's matrix (0..22)
    uint8_t q;      // expert slot
    uint8_t kb0;    // first K-block (even)
    uint8_t nkb;    // K-blocks (even)
    uint8_t flags;  // kFirst: first stage of a segment, kLast: last
    uint8_t pad[3];
};
constexpr uint8_t kFirst = 1;
constexpr uint8_t kLast = 2;
struct PlanSeg {
    uint8_t tile;   // tile of the phase (gate/up: slot * 23 + tile)
    uint8_t mask;   // MMA issuers with K-blocks in the segment
    uint8_t nslot;  // contributors to the tile
    uint8_t slot;   // this CTA's slot; nslot - 1: this CTA reduces the tile
};
struct Plan {
    PlanStage st[kPlanStages];
    PlanSeg seg[kPlanSegs];
    int nst;
    int nseg;
};

struct alignas(1024) Smem {
    uint8_t a[kStages][2][128][128];              // A stages: two boxes of 128 rows x 256 E2M1, swizzled
    uint8_t sfa[kStages][4][kScaleBlockBytes];    // their scale blocks (gate/up: gate 0-1, up 2-3; down: 0-3)
    uint8_t bgu[kBlocks][kBRowBytes];             // gate/up B: digit terms of h
    uint8_t bdown[kDownSlots][kBlocks][kBRowBytes];  // down B: digit terms of w * hidden of this CTA's experts
    alignas(16) uint8_t gcode[kCodeBytes];        // gate/up B block codes
    alignas(16) uint8_t dcode[kDownSlots][kCodeBytes];  // down B block codes
    double rsum[kEpiWarps][kMaxExperts + 1];      // next-layer router sums per epilogue warp
    float own_part[kOwnMax][2][128];              // partials of the tiles this CTA reduces (gate, up)
    Plan plan[kTopK + 1][2];                      // [local experts][phase]
    int dslot[kTopK];                             // expert slot -> bdown slot, -1 if unused
    float logit[kMaxExperts];
    float bound[kMaxExperts];
    float val[kMaxExperts];
    double red[kComputeWarps];
    uint64_t full[kStages];       // a stage's bytes landed
    uint64_t empty[kStages];      // the MMAs of a stage completed
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t sel_full;            // the step's selection is published
    uint64_t setup;               // the down B operands of the step landed
    uint64_t rwbar;               // a down reducer's staged router weights landed
    uint32_t rw_uses;             // stagings consumed so far (its parity), written by thread 0 only
    uint32_t rw_issued;           // stagings issued so far, written by thread 0 only
    uint64_t fin;
    uint32_t tmem;
    int go;      // grid-barrier / end-of-step verdict, written by thread 0 only
    uint32_t seq;  // tag base of this launch, read from the device at the start
    int epi_go;  // epilogue verdict, written by thread 0 only
    int sel[kTopK];
    int local[kTopK];
    int slot_of[kTopK];
    float wts[kTopK];
    int n_local;
    int amb;
    int abort;
    int last;
    float nscale;  // scalar the gate/up partials are multiplied by (the RMSNorm scale; 1 in mode 0)
    int step_layer;  // mode 2: the layer of the step in hand (for the loads warp)
    int srv_layer;   // mode 2: the request's layer, or -1 when the server leaves
    int srv_exit;    // mode 2: the compute group left the step loop (the loads warp follows)
    uint32_t steps_run;  // steps this launch ran (mode 2: requests served), written by thread 0 only
};

static_assert(sizeof(Smem) + 1024 <= 232448, "shared memory per CTA");
// TMA boxes with 128-byte swizzle land on 1024-byte boundaries; bulk copies
// and tcgen05 operand / copy sources need 16-byte alignment.
static_assert(offsetof(Smem, a) % 1024 == 0 && sizeof(Smem::a[0][0]) % 1024 == 0, "A stage alignment");
static_assert(offsetof(Smem, sfa) % 16 == 0 && offsetof(Smem, bgu) % 16 == 0 && offsetof(Smem, bdown) % 16 == 0 &&
                  offsetof(Smem, gcode) % 16 == 0 && offsetof(Smem, dcode) % 16 == 0,
              "bulk-copy destinations");

// Role-local pipeline counters (each role walks the same stage sequence).
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

// ---- tagged words ----
// An f32 in the low half and, in the high half, the tag seq + step + 1 of the
// step that wrote it: one 8-byte access carries both, so a reader that sees
// the tag has the value, and words of other steps or launches never match.
__device__ __forceinline__ uint32_t step_tag(const Smem &s, int step) {
    return s.seq + uint32_t(step) + 1u;
}
__device__ __forceinline__ unsigned long long tagged(uint32_t tag, float v) {
    return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_tagged(unsigned long long *p, unsigned long long w) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Bounded wait; a phase that already completed costs one try_wait.
__device__ __forceinline__ bool wait_bar(Smem &s, uint64_t *bar, uint32_t parity, uint32_t *status) {
    if (tc::mbar_try_wait(bar, parity)) {
        return true;
    }
    if (aborted(s)) {
        return false;
    }
    if (!tc::mbar_wait(bar, parity)) {
        fail_wait(s, status);
        return false;
    }
    return true;
}

// Polls up to N tagged words until each carries `tag`.  Every round issues
// the loads of all words still missing before checking any of them, so their
// round trips to L2 overlap (a word-by-word wait would pay one per word).
// addr(k) is word k's address, `miss` has bit k set for each word to fetch;
// the f32 halves land in v[k].  Bounded: after a timeout or an abort the
// missing values stay as they are, with the status set.
template <int N, bool kSys = false, class F>
__device__ __forceinline__ void poll_tagged(Smem &s, F addr, uint32_t miss, uint32_t tag, float (&v)[N],
                                            uint32_t *status) {
    unsigned long long t0 = 0ull;
    while (miss != 0u) {
        unsigned long long w[N];
#pragma unroll
        for (int k = 0; k < N; ++k) {
            if ((miss >> k) & 1u) {
                if constexpr (kSys) {
                    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w[k]) : "l"(addr(k)) : "memory");
                } else {
                    w[k] = ld_tagged(addr(k));
                }
            } else {
                w[k] = 0ull;
            }
        }
#pragma unroll
        for (int k = 0; k < N; ++k) {
            if (((miss >> k) & 1u) && uint32_t(w[k] >> 32) == tag) {
                v[k] = __uint_as_float(uint32_t(w[k]));
                miss &= ~(1u << k);
            }
        }
        if (miss == 0u || aborted(s)) {
            return;
        }
        const unsigned long long now = tc::now_ns();
        if (t0 == 0ull) {
            t0 = now;
        } else if (now - t0 > kGridWaitNs) {
            fail_wait(s, status);
            return;
        }
    }
}

// ---- expert parallelism: the partial output rows of the ranks ----
// System scope: the words of the exchange buffers are written by other GPUs
// over NVLink (their stores to this GPU's memory) and read here.
__device__ __forceinline__ void st_tagged_sys(unsigned long long *p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// This rank's partial v of output row `row` (the sum over its own selected
// experts) goes to slot [step parity][rank][row] of every other rank's
// exchange buffer; the ranks' partials are then added in rank order, so every
// rank gets the same bits (and so the same next selection).  A rank that
// never writes ends the wait with kStatusWaitTimeout.
__device__ __forceinline__ float exchange_row(Smem &s, const StackArgs &a, int step, int row, float v, uint32_t tag) {
    const size_t par = size_t(step & 1) * size_t(a.world) * kXchRow;
    const unsigned long long word = tagged(tag, v);
    for (int r = 0; r < a.world; ++r) {
        if (r != a.rank) {
            st_tagged_sys(a.xch[r] + par + size_t(a.rank) * kXchRow + row, word);
        }
    }
    const unsigned long long *own = a.xch[a.rank] + par + row;
    float pv[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
        pv[r] = (r == a.rank) ? v : 0.0f;
    }
    const uint32_t others = ((1u << a.world) - 1u) & ~(1u << a.rank);
    poll_tagged<kMaxWorld, true>(s, [&](int r) { return own + size_t(r) * kXchRow; }, others, tag, pv, a.status);
    float tot = pv[0];
#pragma unroll
    for (int r = 1; r < kMaxWorld; ++r) {
        if (r < a.world) {
            tot = __fadd_rn(tot, pv[r]);
        }
    }
    return tot;
}

// Waits (bounded) until the counter at p reaches `want`; acquire.
__device__ __forceinline__ void wait_count(Smem &s, const unsigned *p, unsigned want, uint32_t *status) {
    const unsigned long long t0 = tc::now_ns();
    while (true) {
        unsigned cur;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(p) : "memory");
        if (int(cur - want) >= 0 || aborted(s)) {
            return;
        }
        if (tc::now_ns() - t0 > 2000000000ull) {
            fail_wait(s, status);
            return;
        }
    }
}

// 4-byte asynchronous global -> shared copy (cp.async; any 4-byte aligned
// source), completed by cp.async.wait_all of the issuing thread.
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(tc::smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

// Named barriers of whole warps: bar.sync needs every lane of a warp to
// execute it together, and a warp whose lanes diverged before (one lane
// polling, publishing, ...) would otherwise arrive twice and let the others
// through early, so each warp reconverges first.
__device__ __forceinline__ void epi_sync() {
    __syncwarp();
    asm volatile("bar.sync 2, 128;" ::: "memory");
}

__device__ __forceinline__ void compute_sync() {
    __syncwarp();
    asm volatile("bar.sync 1, %0;" ::"n"(kComputeThreads) : "memory");
}

// Bounded grid barrier of the compute groups.  bar[0] counts arrivals over
// the whole launch (zeroed by the host before it); barrier n completes when
// it reaches n * gridDim.x.
__device__ bool grid_barrier(unsigned *bar, unsigned &gen, uint32_t *status, Smem &s) {
    compute_sync();
    if (threadIdx.x == 0 && !aborted(s)) {
        gen += 1u;
        const unsigned target = gen * gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const unsigned long long t0 = tc::now_ns();
        while (true) {
            unsigned cur;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(bar) : "memory");
            if (int(cur - target) >= 0) {
                break;
            }
            if (tc::now_ns() - t0 > kGridWaitNs) {
                fail_wait(s, status);
                break;
            }
        }
    }
    if (threadIdx.x == 0) {
        s.go = aborted(s) ? 0 : 1;
    }
    compute_sync();
    return s.go != 0;
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Step stamps for profiling (thread 0 of CTA 0; points 8 and 9 = latest
// phase-B / phase-C end over CTAs).
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

// Contiguous unit range of CTA c out of g over `units` units (c * units and
// u * g stay below 2^31: g <= 1024 CTAs, units <= 2^20).
__device__ __forceinline__ int range_lo(int c, int g, int units) {
    return int(unsigned(c) * unsigned(units) / unsigned(g));
}

// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of(int u, int g, int units) {
    int c = int(unsigned(u) * unsigned(g) / unsigned(units));
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
    int kunits;  // K-units (K-block pairs) per tile: 45 for gate/up, n_local * 45 for down
};

__device__ __forceinline__ Phase gateup_phase(int n_local) {
    return Phase{0, n_local * kTiles, kPairs};
}

__device__ __forceinline__ Phase down_phase(int n_local) {
    return Phase{1, kTiles, n_local * kPairs};
}

struct Ctx {
    const StackArgs *a;
    const StackLayer *L;
    Smem *s;
    uint32_t tbase;
};

// What one stage holds.  Gate/up: K-blocks of one aligned group of 8 (one
// weight box), gate rows in box 0 and up rows in box 1.  Down: K-blocks of
// one aligned group of 16, K-blocks 8b..8b+7 in box b & 1.

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void bulk_load_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            tc::smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(tc::smem_u32(bar)), "l"(pol)
        : "memory");
}

// ---- loads (warp 9, lane 0) ----
// Expert weights are read once per token: they go through L2 as evict-first,
// so they do not push out the partials, operands and code the step reuses.
__device__ bool produce_phase(const Ctx &c, const Plan &pl, int kind, const int (&le)[kTopK], Pipe &pp) {
    Smem &s = *c.s;
    const TmaDesc *tm = c.L->tma;
    const uint8_t *gate = c.L->gate;
    const uint8_t *up = c.L->up;
    const uint8_t *down = c.L->down;
    const uint64_t pol = tc::policy_evict_first();
    for (int si = 0; si < pl.nst; ++si) {
        const PlanStage r = pl.st[si];
        const uint32_t st = pp.stage % kStages;
        const uint32_t use = pp.stage / kStages;
        if (use > 0 && !wait_bar(s, &s.empty[st], (use - 1) & 1, c.a->status)) {
            return false;
        }
        // the step's first gate/up stages go out two at a time: later ones
        // wait until the one two before has landed
        if (kind == 0 && si >= 2 && si < kStages) {
            const uint32_t prev = pp.stage - 2;
            if (!wait_bar(s, &s.full[prev % kStages], (prev / kStages) & 1, c.a->status)) {
                return false;
            }
        }
        const int e = (r.q == 0) ? le[0] : (r.q == 1) ? le[1] : (r.q == 2) ? le[2] : le[3];
        const int c0 = r.kb0 >> 2;
        const int c1 = (r.kb0 + r.nkb - 1) >> 2;
        const uint32_t nc = uint32_t(c1 - c0 + 1);
        const int row0 = 128 * r.tile;
        const size_t so = size_t(e) * kPackedMatrixBytes + scale_block_offset(r.tile, c0);
        if (kind == 0) {
            const int x = 16 * (r.kb0 & ~7);  // byte offset of the stage's box in a row
            tc::mbar_expect_tx(&s.full[st], 2 * kBoxTx + 2 * nc * uint32_t(kScaleBlockBytes));
            tc::tma_load_3d_hint(&s.a[st][0][0][0], tm + kTmaGate, x, row0, e, &s.full[st], pol);
            tc::tma_load_3d_hint(&s.a[st][1][0][0], tm + kTmaUp, x, row0, e, &s.full[st], pol);
            bulk_load_hint(&s.sfa[st][c0 & 1][0], gate + so, nc * kScaleBlockBytes, &s.full[st], pol);
            bulk_load_hint(&s.sfa[st][2 + (c0 & 1)][0], up + so, nc * kScaleBlockBytes, &s.full[st], pol);
        } else {
            const int b0 = r.kb0 >> 3;
            const int b1 = (r.kb0 + r.nkb - 1) >> 3;
            tc::mbar_expect_tx(&s.full[st], uint32_t(b1 - b0 + 1) * kBoxTx + nc * uint32_t(kScaleBlockBytes));
            for (int b = b0; b <= b1; ++b) {
                tc::tma_load_3d_hint(&s.a[st][b & 1][0][0], tm + kTmaDown, 128 * b, row0, e, &s.full[st], pol);
            }
            bulk_load_hint(&s.sfa[st][c0 & 3][0], down + so, nc * kScaleBlockBytes, &s.full[st], pol);
        }
        ++pp.stage;
    }
    return true;
}

// Issuers that have K-blocks in a segment of phase p: issuer k owns, in each
// stage, scale chunk k & 1 of the gate (k < 2) or up (k >= 2) box, or chunk k
// of the four of a down stage.  units [u_lo, u_hi) of tile `tile`.
__device__ __forceinline__ uint32_t segment_issuers(const Phase &p, int tile, int u_lo, int u_hi) {
    uint32_t mask = 0;
    for (int u = u_lo; u < u_hi; ++u) {
        const int pr = (u - tile * p.kunits) % kPairs;
        if (p.kind == 0) {
            mask |= ((pr >> 1) & 1) ? 0xAu : 0x5u;
        } else {
            mask |= 1u << ((pr >> 1) & 3);
        }
    }
    return mask;
}

// ---- MMA issuers (warps 4-7, lane 0; issuer k = warp - 4) ----
__device__ void run_mma(const Ctx &c, const Plan &pl, int kind, Pipe &pp, int k) {
    Smem &s = *c.s;
    const uint32_t a0 = tc::smem_u32(&s.a[0][0][0][0]);
    const uint32_t sf0 = tc::smem_u32(&s.sfa[0][0][0]);
    const uint32_t tbase = c.tbase;
    uint32_t db = 0;
    bool first = true;
    for (int si = 0; si < pl.nst; ++si) {
        const PlanStage r = pl.st[si];
        if (r.flags & kFirst) {
            db = pp.seg & 1;
            const uint32_t duse = pp.seg >> 1;
            if (duse > 0 && !wait_bar(s, &s.acc_empty[db], (duse - 1) & 1, c.a->status)) {
                return;
            }
            tc::fence_after_sync();
            first = true;
        }
        const uint32_t st = pp.stage % kStages;
        if (!wait_bar(s, &s.full[st], (pp.stage / kStages) & 1, c.a->status)) {
            return;
        }
        tc::fence_after_sync();
        // this issuer's scale chunk of the stage and its K-blocks in it
        const int m = (kind == 0) ? (k >> 1) : 0;
        const int chunk = (kind == 0) ? ((r.kb0 & ~7) >> 2) + (k & 1) : ((r.kb0 & ~15) >> 2) + k;
        const int lo = max(r.kb0, 4 * chunk);
        const int hi = min(r.kb0 + r.nkb, 4 * chunk + 4);
        if (lo < hi) {
            const uint32_t abase = a0 + st * uint32_t(sizeof(s.a[0]));
            const uint32_t sfa = tbase + kColSfa + 16 * st + 4 * uint32_t(k);
            tc::sf_copy(sfa, sf0 + st * uint32_t(sizeof(s.sfa[0])) + kScaleBlockBytes * uint32_t(k));
            const uint32_t dcol = tbase + kColD + 64 * db + 16 * uint32_t(k);
            uint32_t bbase, sfb0;
            if (kind == 0) {
                bbase = tc::smem_u32(&s.bgu[0][0]);
                sfb0 = tbase + kColSfbG;
            } else {
                const int ds = s.dslot[r.q];
                bbase = tc::smem_u32(&s.bdown[ds][0][0]);
                sfb0 = tbase + kColSfbD + kSfbCols * uint32_t(ds);
            }
            for (int kb = lo; kb < hi; kb += 2) {
                const uint32_t sel = uint32_t(kb & 3);
                const uint32_t box = (kind == 0) ? uint32_t(m) : uint32_t((kb >> 3) & 1);
                const uint32_t aoff = 16384u * box + 32u * uint32_t((kb >> 1) & 3);
                const uint64_t bd = tc::smem_desc(bbase + uint32_t(kb) * kBRowBytes, kBRowBytes, 128);
                tc::mma_f4(dcol, tc::smem_desc_sw128(abase + aoff), bd, tc::instr_desc_f4(kN, sel), sfa | (sel << 30),
                           (sfb0 + 4 * uint32_t(kb >> 2)) | (sel << 30), !first);
                first = false;
            }
        }
        tc::mma_commit(&s.empty[st]);
        ++pp.stage;
        if (r.flags & kLast) {
            tc::mma_commit(&s.acc_full[db]);
            ++pp.seg;
        }
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

// The plan of phase p for this CTA (one thread).  Segments (one per tile the
// CTA's unit range touches) go from the last to the first: the last one is
// the head of a tile a later CTA reduces, so its partial is published first,
// and the first one -- the tail of a tile this CTA reduces -- comes last,
// when the earlier CTA's partial of that tile (its first segment) is already
// out.  Stages within a segment go in K order; a stage spans one aligned
// group of 4 (gate/up) or 8 (down) K-block pairs.
__device__ void build_plan(Plan &pl, const Phase &p, uint32_t *status) {
    const int units = p.tiles * p.kunits;
    const int u0 = range_lo(blockIdx.x, gridDim.x, units);
    const int span = (p.kind == 0) ? 4 : 8;  // pairs
    int nst = 0, nseg = 0;
    for (int seg_end = range_lo(blockIdx.x + 1, gridDim.x, units); seg_end > u0;) {
        const int tile = (seg_end - 1) / p.kunits;
        const int seg_lo = max(u0, tile * p.kunits);
        if (nseg < kPlanSegs) {
            int n, slot;
            tile_slots(p, tile, n, slot);
            PlanSeg &g = pl.seg[nseg];
            g.tile = uint8_t(tile);
            g.mask = uint8_t(segment_issuers(p, tile, seg_lo, seg_end));
            g.nslot = uint8_t(min(n, 255));
            g.slot = uint8_t(slot);
        }
        ++nseg;
        uint8_t flags = kFirst;
        for (int u = seg_lo; u < seg_end;) {
            const int ku0 = u - tile * p.kunits;
            int q = ku0 / kPairs;
            const int pr = ku0 - q * kPairs;
            int t = tile;
            if (p.kind == 0) {
                q = tile / kTiles;
                t = tile - q * kTiles;
            }
            const int np = min(min((pr & ~(span - 1)) + span, kPairs) - pr, seg_end - u);
            u += np;
            if (nst < kPlanStages) {
                PlanStage &r = pl.st[nst];
                r.tile = uint8_t(t);
                r.q = uint8_t(q);
                r.kb0 = uint8_t(2 * pr);
                r.nkb = uint8_t(2 * np);
                r.flags = uint8_t(flags | (u == seg_end ? kLast : 0));
            }
            ++nst;
            flags = 0;
        }
        seg_end = seg_lo;
    }
    if (nst > kPlanStages || nseg > kPlanSegs) {
        set_status(status, kStatusBadShape);
    }
    pl.nst = min(nst, kPlanStages);
    pl.nseg = min(nseg, kPlanSegs);
}

// tagged_sum of the gate (p) and up (p + 128) partials together: four
// contributors (eight words) per batch, their polls in flight together.
__device__ __forceinline__ void tagged_sum2(Smem &s, const unsigned long long *p, size_t stride, int nslot, float &g,
                                            float &u, uint32_t tag, uint32_t *status) {
    constexpr int kBatch = 4;
    float sg = 0.0f, su = 0.0f;
    for (int k0 = 0; k0 + 1 < nslot; k0 += kBatch) {
        float v[2 * kBatch];
        uint32_t want = 0u;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            v[2 * j] = v[2 * j + 1] = 0.0f;
            want |= (k0 + j + 1 < nslot) ? (3u << (2 * j)) : 0u;
        }
        poll_tagged<2 * kBatch>(
            s, [&](int k) { return p + size_t(k0 + (k >> 1)) * stride + 128 * (k & 1); }, want, tag, v, status);
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (k0 + j + 1 < nslot) {
                sg += v[2 * j];
                su += v[2 * j + 1];
            }
        }
    }
    g = sg + g;
    u = su + u;
}

// Tagged partials of tile `tile` in phase p of `step`: [slot][256 or 128].
__device__ __forceinline__ size_t part_stride(const Phase &p) {
    return (p.kind == 0) ? 256 : 128;
}
__device__ __forceinline__ unsigned long long *part_base(const StackArgs &a, const Phase &p, int step, int tile) {
    return (p.kind == 0 ? a.part_gu + size_t(step & 1) * (kPartGuWords / 2)
                        : a.part_dn + size_t(step & 1) * (kPartDnWords / 2)) +
           size_t(tile) * kMaxSlots * part_stride(p);
}

// Sum over the contributors in slot order; this CTA reduces the tile, so its
// own partial `mine` is the last one.  p: this row's word of slot 0.
// Eight contributors per batch, their polls in flight together.
__device__ __forceinline__ float tagged_sum(Smem &s, const unsigned long long *p, size_t stride, int nslot, float mine,
                                            uint32_t tag, uint32_t *status) {
    constexpr int kBatch = 8;
    float sum = 0.0f;
    for (int k0 = 0; k0 + 1 < nslot; k0 += kBatch) {
        float v[kBatch];
        uint32_t want = 0u;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            v[j] = 0.0f;
            want |= (k0 + j + 1 < nslot) ? (1u << j) : 0u;
        }
        poll_tagged<kBatch>(s, [&](int k) { return p + size_t(k0 + k) * stride; }, want, tag, v, status);
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (k0 + j + 1 < nslot) {
                sum += v[j];
            }
        }
    }
    return sum + mine;
}

// Sums v[0..15] over the warp's 32 lanes: afterwards lane l holds the total of
// value 8*b4 + 4*b3 + 2*b2 + b1 (b = bits of l), identical in lanes l and l^1.
__device__ __forceinline__ float transpose_sum16(float (&v)[16], int lane) {
#pragma unroll
    for (int lvl = 0; lvl < 4; ++lvl) {
        const int off = 16 >> lvl;
        const int half = 8 >> lvl;
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j < half) {
                const float send = upper ? v[j] : v[j + half];
                const float keep = upper ? v[j + half] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

__device__ __forceinline__ int transpose_index(int lane) {
    return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// ---- epilogue warps (0-3): one thread per tile row ----
// Every contributor to a tile but the last publishes its partial as tagged
// words and moves on; the last contributor -- the CTA holding the tile's last
// units -- reduces: it polls the words, sums the partials in slot order and
// finishes the tile.  A CTA first reads all of its segments (so its partials
// for other tiles go out at once), then reduces the tiles it owns.
struct EpiTile {
    int tile;
    int nslot;
    int slot;
};

// Operands of a tile's epilogue, loaded before the tile's accumulators are.
struct TileOps {
    float bias_g, bias_u;  // gate/up: biases of this row
    float bsum;            // down: sum_q w_q b_q of this row
    float resid;           // down: residual
    float nw;              // down: next layer's RMSNorm weight
    float xnext;           // down: next token's input (last layer)
    float rw[kPreE];       // down: next layer's router weights of this row
};

// Steps per token of a launch: its layers, or 1 in the server mode (each
// request is one step on its own layer).
__device__ __forceinline__ int steps_per_token(const StackArgs &a) {
    return a.mode == 2 ? 1 : a.layer_end - a.layer_begin;
}

// Loads of a tile's epilogue operands, issued where they stand: as volatile
// asm they stay ahead of the accumulator waits that follow them (a plain load
// of read-only data may be moved down to its first use, which would put a
// memory round trip on the reducer's critical path).
__device__ __forceinline__ float ld_early_nc(const float *p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_early_cg(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

template <bool kWideRouter>
__device__ __forceinline__ void load_tile_ops(const Ctx &c, const Phase &p, int tile, int t_token, int li, bool next_router,
                                              TileOps &o) {
    const Smem &s = *c.s;
    const StackArgs &a = *c.a;
    const StackLayer &L = *c.L;
    const int i = threadIdx.x;
    const int nl = a.layer_end - a.layer_begin;
    const bool more_layers = (li + 1 < nl);
    o.bias_g = o.bias_u = o.bsum = o.resid = o.nw = o.xnext = 0.0f;
#pragma unroll
    for (int e = 0; e < kPreE; ++e) {
        o.rw[e] = 0.0f;
    }
    if (p.kind == 0) {
        const int q = tile / kTiles;
        const int row = 128 * (tile - q * kTiles) + i;
        if (row < kDim) {
            const int le = s.local[s.slot_of[q]];
            o.bias_g = __ldg(L.gate_b + size_t(le) * kDim + row);
            o.bias_u = __ldg(L.up_b + size_t(le) * kDim + row);
        }
        return;
    }
    const int row = 128 * tile + i;
    if (kWideRouter && next_router) {
        // the next layer's router weights of this tile's rows for the experts
        // past kPreE (staged by the reducer after the exchange, when the sums
        // are on the step's critical path) go to L2 now: one tensor prefetch
        // of the box the staging copies
        if (i == 0) {
            const StackLayer &N = a.layers[more_layers ? a.layer_begin + li + 1 : a.layer_begin];
            tc::tma_prefetch_2d(N.tma + kTmaRouter, 128 * tile, kPreE);
        }
    }
    if (row >= kDim) {
        return;
    }
    float b[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        b[k] = (k < s.n_local) ? ld_early_nc(L.down_b + size_t(s.local[s.slot_of[k]]) * kDim + row) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        if (k < s.n_local) {
            o.bsum = __fadd_rn(o.bsum, __fmul_rn(s.wts[s.slot_of[k]], b[k]));
        }
    }
    if (a.mode == 1) {
        const int tr = t_token & a.row_mask;
        const float *xcur = (li == 0) ? a.x + size_t(tr) * kDim : a.y + size_t(tr) * kDim;
        o.resid = ld_early_cg(xcur + row);
    }
    if (next_router) {
        const StackLayer &N = a.layers[more_layers ? a.layer_begin + li + 1 : a.layer_begin];
        const float *nrw = N.router_w;
        o.nw = ld_early_nc(N.norm_w + row);
        if (!more_layers) {
            o.xnext = ld_early_cg(a.x + size_t(t_token + 1) * kDim + row);
        }
        static_assert(kPreE <= 32, "every handle has at least kPreE experts (32 or 128)");
#pragma unroll
        for (int e = 0; e < kPreE; ++e) {
            o.rw[e] = ld_early_nc(nrw + size_t(e) * kDim + row);
        }
    }
}

// The tile's epilogue proper (reducer only): gate/up -> SwiGLU, routing
// weight and the digit terms of the down projection's input; down -> bias,
// residual, output rows and the next layer's router sums.
template <bool kWideRouter>
__device__ void finish_tile(const Ctx &c, const Phase &p, const EpiTile &et, const TileOps &o, float pg, float pu,
                            int t_token, int li, bool next_router) {
    Smem &s = *c.s;
    const StackArgs &a = *c.a;
    const int i = threadIdx.x;
    const int w = i >> 5;
    const int lane = i & 31;
    const int E = a.experts;
    const int nl = steps_per_token(a);
    const bool more_layers = (li + 1 < nl);
    const int tile = et.tile;
    const int step = t_token * nl + li;
    const uint32_t tag = step_tag(s, step);
    // down with the next router: the router weights of this tile's rows for
    // the experts past kPreE (warm in L2 from load_tile_ops) go into the stage
    // ring, idle until this CTA publishes the next selection, one bulk copy per
    // expert, while the partials below are summed
    const bool stage_rw = kWideRouter && p.kind == 1 && next_router;
    const uint32_t rw_parity = kWideRouter ? (s.rw_uses & 1u) : 0u;
    if (stage_rw && i == 0) {
        // one tensor copy: [E - kPreE experts][128 rows] f32 (rows past 2880
        // read as zero), the layout the products below index
        const StackLayer &N = a.layers[more_layers ? a.layer_begin + li + 1 : a.layer_begin];
        ++s.rw_issued;
        tc::mbar_expect_tx(&s.rwbar, uint32_t(E - kPreE) * 128u * 4u);
        tc::tma_load_2d(&s.a[0][0][0][0], N.tma + kTmaRouter, 128 * tile, kPreE, &s.rwbar);
    }
    if (et.nslot > 1) {
        // the other contributors' tagged partials (after an abort the sums
        // are garbage; every later wait returns at once)
        const unsigned long long *base = part_base(a, p, step, tile) + i;
        if (p.kind == 0) {
            tagged_sum2(s, base, part_stride(p), et.nslot, pg, pu, tag, a.status);
        } else {
            pg = tagged_sum(s, base, part_stride(p), et.nslot, pg, tag, a.status);
        }
    }
    if (p.kind == 0) {
        const int q = tile / kTiles;
        const int row = 128 * (tile - q * kTiles) + i;
        // warp w holds K-block (row >> 5) of the down projection's input
        if (row - lane < kDim) {
            float h = 0.0f;
            if (row < kDim) {
                const float gv = __fadd_rn(o.bias_g, __fmul_rn(pg, s.nscale));
                const float uv = __fadd_rn(o.bias_u, __fmul_rn(pu, s.nscale));
                h = __fmul_rn(swiglu_ref(gv, uv), s.wts[s.slot_of[q]]);
            }
            const int kb = row >> 5;
            uint8_t *bd = a.bdown + size_t(step & 1) * (kBdownBytes / 2);
            const uint32_t code = tc::digit_split_store(h, bd + (size_t(q) * kBlocks + kb) * kBRowBytes, lane);
            if (lane == 0) {
                a.sfb_down[size_t(step & 1) * (kSfbDownBytes / 2) + size_t(q) * kCodeBytes + kb] = uint8_t(code);
            }
        }
        // this tile of expert slot q is in place for the down phase
        epi_sync();
        if (i == 0) {
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.cnt_b + q) : "memory");
        }
        return;
    }
    const int row = 128 * tile + i;
    float yv = 0.0f;
    if (row < kDim) {
        float out = __fadd_rn(pg, o.bsum);
        if (a.world > 1) {
            out = exchange_row(s, a, step, row, out, tag);
        }
        yv = (a.mode == 1) ? __fadd_rn(o.resid, out) : out;
        if (a.ylog && step < a.log_steps) {
            a.ylog[size_t(step) * kDim + row] = yv;
        }
    }
    if (!next_router && row < kDim) {
        a.y[size_t(t_token & a.row_mask) * kDim + row] = yv;
    }
    if (!next_router && a.mode == 2 && row < kDim) {
        // the server's row goes straight to the mailbox in host memory, tagged
        // with the request's number (the host polls the words themselves)
        const unsigned long long w = tagged(a.mbox_base + uint32_t(step) + 1u, yv);
        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a.mbox->y + row), "l"(w) : "memory");
    }
    if (next_router) {
        // router sums of the next (token, layer) over these rows: per warp,
        // f32 products transposed-summed over the 32 rows (f64 from there on)
        const float xr = more_layers ? yv : o.xnext;
        const float xg = __fmul_rn(xr, o.nw);  // 0 past the last row
        // 16 experts' products of this row -> their sums over the warp's rows
        const auto route16 = [&](float (&v)[16], int b) {
            const float tot = transpose_sum16(v, lane);
            const int e = 16 * b + transpose_index(lane);
            if ((lane & 1) == 0 && e < E) {
                s.rsum[w][e] = double(tot);
            }
        };
        // the first kPreE experts from registers (static indices: o.rw stays
        // in registers)
        static_assert(kPreE == 32, "two groups of 16 preloaded experts");
        {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                v[j] = __fmul_rn(o.rw[j], xg);
            }
            route16(v, 0);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                v[j] = __fmul_rn(o.rw[16 + j], xg);
            }
            route16(v, 1);
        }
        if (kWideRouter) {
            // every thread waits for the staged weights (bounded, and not cut
            // short by an abort; a wait that gives up leaves the copies to
            // the drain before the CTA exits)
            if (!tc::mbar_wait(&s.rwbar, rw_parity)) {
                fail_wait(s, a.status);
            }
            const float *rws = reinterpret_cast<const float *>(&s.a[0][0][0][0]);
            for (int b = kPreE / 16; 16 * b < E; ++b) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int e = 16 * b + j;
                    v[j] = (e < E && row < kDim) ? __fmul_rn(rws[size_t(e - kPreE) * 128 + i], xg) : 0.0f;
                }
                route16(v, b);
            }
        }
        const double sq = warp_sum_d(row < kDim ? double(__fmul_rn(xr, xr)) : 0.0);
        if (lane == 0) {
            s.rsum[w][E] = sq;
        }
        if (stage_rw) {
            // the ring's next writers are bulk copies and TMA loads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        epi_sync();
        if (stage_rw && i == 0) {
            ++s.rw_uses;
        }
        // this tile's router sums for the next step, first: each f64 as two
        // tagged f32 words (hi, then the remainder) that every CTA polls
        unsigned long long *rp = a.rpt + (size_t(step & 1) * kTiles + tile) * (kMaxExperts + 1) * 2;
        for (int e = i; e < E + 1; e += 32 * kEpiWarps) {
            double tot = 0.0;
#pragma unroll
            for (int k = 0; k < kEpiWarps; ++k) {
                tot += s.rsum[k][e];
            }
            const float hi = __double2float_rn(tot);
            const float lo = __double2float_rn(tot - double(hi));
            // both words in one 16-byte store (each half is single-copy atomic
            // and carries the tag)
            asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(rp + 2 * e), "l"(tagged(tag, hi)),
                         "l"(tagged(tag, lo))
                         : "memory");
        }
        // then this tile's output rows and the next step's gate/up B operand
        // (digit terms of x * g; the RMSNorm scale is a scalar applied to the
        // products), counted on their own
        if (row < kDim) {
            a.y[size_t(t_token & a.row_mask) * kDim + row] = yv;
        }
        // the next step's gate/up B operand: digit terms of x * g (the RMSNorm
        // scale is a scalar applied to the products)
        if (row - lane < kDim) {
            const int kb = row >> 5;
            uint8_t *bn = a.bnext + size_t(step & 1) * (kBnextBytes / 2);
            const uint32_t code = tc::digit_split_store(xg, bn + size_t(kb) * kBRowBytes, lane);
            if (lane == 0) {
                a.bnext_code[size_t(step & 1) * (kBnextCodeBytes / 2) + kb] = uint8_t(code);
            }
        }
        epi_sync();  // also: s.rsum is read before this CTA's next tile rewrites it
        if (i == 0) {
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.cnt_y) : "memory");
        }
    }
}

template <bool kWideRouter>
__device__ void run_epilogue(const Ctx &c, const Phase &p, const Plan &pl, Pipe &pp, int t_token, int li,
                             bool next_router) {
    Smem &s = *c.s;
    const StackArgs &a = *c.a;
    const int i = threadIdx.x;  // 0..127: tile row
    const int w = i >> 5;
    // The first tile this CTA reduces (in plan order) has its operands loaded
    // now, while the MMAs run.
    int first_owned = -1;
    for (int g = pl.nseg - 1; g >= 0; --g) {
        if (pl.seg[g].slot + 1 == pl.seg[g].nslot) {
            first_owned = pl.seg[g].tile;
        }
    }
    const int step = t_token * steps_per_token(a) + li;
    const uint32_t tag = step_tag(s, step);
    TileOps ops;
    if (first_owned >= 0) {
        load_tile_ops<kWideRouter>(c, p, first_owned, t_token, li, next_router, ops);
    }
    EpiTile own[kOwnMax];
    int nown = 0;
    for (int g = 0; g < pl.nseg; ++g) {
        const PlanSeg sg = pl.seg[g];
        const int tile = sg.tile;
        const uint32_t mask = sg.mask;
        const uint32_t db = pp.seg & 1;
        const uint32_t duse = pp.seg >> 1;
        ++pp.seg;
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
        // the issuers' accumulators (gate/up: issuers 0-1 gate, 2-3 up), term
        // partials smallest digit first, issuers in order
        float pg = 0.0f, pu = 0.0f;
#pragma unroll 1
        for (int k = 0; k < kIssuers; ++k) {
            if (mask & (1u << k)) {
                float d[16];
                tc::tmem_ld16(c.tbase + (uint32_t(32 * w) << 16) + kColD + 64 * db + 16 * k, d);
                tc::wait_ld();
                float part = 0.0f;
#pragma unroll
                for (int n = 0; n < tc::kDigitTerms; ++n) {
                    part += d[n];
                }
                if (p.kind == 0 && k >= 2) {
                    pu += part;
                } else {
                    pg += part;
                }
            }
        }
        tc::fence_before_sync();
        mbar_arrive(&s.acc_empty[db]);
        EpiTile et;
        et.tile = tile;
        et.nslot = sg.nslot;
        et.slot = sg.slot;
        if (et.nslot > kMaxSlots) {
            if (i == 0) {
                set_status(a.status, kStatusBadShape);
            }
            continue;
        }
        if (et.slot == et.nslot - 1) {
            // this CTA reduces the tile: keep the partial for later
            if (nown < kOwnMax) {
                s.own_part[nown][0][i] = pg;
                s.own_part[nown][1][i] = pu;
#pragma unroll
                for (int k = 0; k < kOwnMax; ++k) {
                    if (k == nown) {
                        own[k] = et;
                    }
                }
                ++nown;
            } else if (i == 0) {
                set_status(a.status, kStatusBadShape);
            }
            continue;
        }
        unsigned long long *base = part_base(a, p, step, tile) + size_t(et.slot) * part_stride(p);
        st_tagged(base + i, tagged(tag, pg));
        if (p.kind == 0) {
            st_tagged(base + 128 + i, tagged(tag, pu));
        }
    }
#pragma unroll
    for (int k = 0; k < kOwnMax; ++k) {
        if (k >= nown) {
            break;
        }
        if (own[k].tile != first_owned) {
            load_tile_ops<kWideRouter>(c, p, own[k].tile, t_token, li, next_router, ops);
        }
        finish_tile<kWideRouter>(c, p, own[k], ops, s.own_part[k][0][i], s.own_part[k][1][i], t_token, li, next_router);
        if (aborted(s)) {
            return;
        }
    }
    if (p.kind == 1 && p.kunits == 0 && int(blockIdx.x) < kTiles) {
        // no selected expert is this rank's (expert parallelism): CTA t still
        // reduces down tile t, with a zero partial, for the exchange and the
        // rows, router sums and B operand that follow it
        load_tile_ops<kWideRouter>(c, p, int(blockIdx.x), t_token, li, next_router, ops);
        EpiTile et;
        et.tile = int(blockIdx.x);
        et.nslot = 1;
        et.slot = 0;
        finish_tile<kWideRouter>(c, p, et, ops, 0.0f, 0.0f, t_token, li, next_router);
    }
}

// Stack mode, step > 0: the router sums of `step`, written by the down
// reducers of the previous step as tagged words (two per f64).  The compute
// threads share the (tile, expert) items -- a few each, their polls in flight
// together -- and park the values in shared memory (the two B-operand areas,
// idle between the previous step's last MMA and this step's operand copies);
// then thread e <= E adds expert e's 23 tile partials in tile
// order (every CTA gets the same sums) into s.rsum[0][e].  Called by every
// compute thread; needs a compute_sync before s.rsum is read.
// kItems (tile, expert) items per thread cover all of them in one round of
// polls: 3 for 32 experts (23 x 33 <= 288 x 3), 11 for 128 (23 x 129 <= 288 x 11).
template <int kItems>
__device__ __forceinline__ void gather_router_sums(Smem &s, const StackArgs &a, int step, int E) {
    static_assert(offsetof(Smem, bdown) == offsetof(Smem, bgu) + sizeof(Smem::bgu) &&
                      sizeof(Smem::bgu) + sizeof(Smem::bdown) >= sizeof(double) * kTiles * (kMaxExperts + 1),
                  "router scratch: the two B-operand areas, adjacent");
    const int ct = threadIdx.x;
    const int per = E + 1;
    const int items = kTiles * per;  // <= kComputeThreads * kItems (checked by the caller)
    const uint32_t tag = step_tag(s, step - 1);
    const unsigned long long *rp = a.rpt + size_t((step - 1) & 1) * kTiles * (kMaxExperts + 1) * 2;
    double *rs = reinterpret_cast<double *>(&s.bgu[0][0]);
    // item i = (tile, expert): its two tagged words (hi, lo) are adjacent and
    // 16-byte aligned, so one vector load fetches both (each 8-byte half is
    // single-copy atomic and carries its own tag)
    const unsigned long long *addr[kItems];
    uint32_t miss = 0u;
#pragma unroll
    for (int m = 0; m < kItems; ++m) {
        const int i = ct + kComputeThreads * m;
        const int t = i / per;
        addr[m] = rp + (size_t(t) * (kMaxExperts + 1) + size_t(i - t * per)) * 2;
        miss |= (i < items) ? (1u << m) : 0u;
    }
    double v[kItems];
    unsigned long long t0 = 0ull;
    while (miss != 0u) {
        unsigned long long w0[kItems], w1[kItems];
#pragma unroll
        for (int m = 0; m < kItems; ++m) {
            w0[m] = w1[m] = 0ull;
            if ((miss >> m) & 1u) {
                asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];"
                             : "=l"(w0[m]), "=l"(w1[m])
                             : "l"(addr[m])
                             : "memory");
            }
        }
#pragma unroll
        for (int m = 0; m < kItems; ++m) {
            if (((miss >> m) & 1u) && uint32_t(w0[m] >> 32) == tag && uint32_t(w1[m] >> 32) == tag) {
                v[m] = double(__uint_as_float(uint32_t(w0[m]))) + double(__uint_as_float(uint32_t(w1[m])));
                miss &= ~(1u << m);
            }
        }
        if (miss == 0u || aborted(s)) {
            break;
        }
        const unsigned long long now = tc::now_ns();
        if (t0 == 0ull) {
            t0 = now;
        } else if (now - t0 > kGridWaitNs) {
            fail_wait(s, a.status);
            break;
        }
    }
#pragma unroll
    for (int m = 0; m < kItems; ++m) {
        const int i = ct + kComputeThreads * m;
        if (i < items) {
            rs[i] = ((miss >> m) & 1u) ? 0.0 : v[m];
        }
    }
    compute_sync();
    if (ct <= E) {
        double sum = 0.0;
        for (int t = 0; t < kTiles; ++t) {
            sum += rs[t * per + ct];
        }
        s.rsum[0][ct] = sum;
    }
    // the areas' next writers: the gate/up operand copy, then the down
    // operand's bulk copies (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void gather_next_operand(Smem &s, const StackArgs &a, int step) {
    const int ct = threadIdx.x;
    if (ct == 0) {
        wait_count(s, a.cnt_y, unsigned(kTiles) * unsigned(step), a.status);
    }
    compute_sync();
    const size_t par = size_t((step - 1) & 1);
    constexpr int kVec = kBlocks * kBRowBytes / 16;
    constexpr int kVecPer = (kVec + kComputeThreads - 1) / kComputeThreads;
    const uint4 *bn = reinterpret_cast<const uint4 *>(a.bnext + par * (kBnextBytes / 2));
    uint4 bv[kVecPer];
#pragma unroll
    for (int k = 0; k < kVecPer; ++k) {
        const int idx = ct + k * kComputeThreads;
        bv[k] = (idx < kVec) ? __ldcg(bn + idx) : make_uint4(0u, 0u, 0u, 0u);
    }
    const uint32_t *bc = reinterpret_cast<const uint32_t *>(a.bnext_code + par * (kBnextCodeBytes / 2));
    const uint32_t code4 = (ct < kCodeBytes / 4) ? __ldcg(bc + ct) : 0u;
    uint4 *dst = reinterpret_cast<uint4 *>(&s.bgu[0][0]);
#pragma unroll
    for (int k = 0; k < kVecPer; ++k) {
        const int idx = ct + k * kComputeThreads;
        if (idx < kVec) {
            dst[idx] = bv[k];
        }
    }
    if (ct < kCodeBytes / 4) {
        reinterpret_cast<uint32_t *>(s.gcode)[ct] = code4;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // s.bgu is read by the MMAs
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

// Order key of a logit: larger logits larger, -0 and +0 equal, NaN below
// every number (INT_MIN, which no number maps to).
__device__ __forceinline__ int logit_key(float v) {
    int b = __float_as_int(v + 0.0f);
    b = (b >= 0) ? b : (b ^ 0x7fffffff);
    return (v == v) ? b : int(0x80000000u);
}

// Top-4 of s.logit, by warp 0, in four rounds of warp reductions: lane l holds
// experts l, l + 32, l + 64, l + 96; each round takes the largest key still in
// play (redux.sync max), then the lowest expert index among its holders
// (redux.sync min), writes it to s.sel[round] and retires it.  The order --
// larger logits first, the lower index first among equal logits, NaN after
// every number -- is the selection sort's with a strict ">"
// (src/model.cpp:296-309) whenever the logits are distinct; equal logits are
// the ambiguous case the callers resolve.  With at least kTopK experts every
// round finds one.
__device__ __forceinline__ void warp_top4(Smem &s, int experts) {
    const int lane = threadIdx.x & 31;
    static_assert(kMaxExperts == 128, "four experts per lane");
    int key[4];
    unsigned live = 0u;  // bit k: expert lane + 32 k is present and not yet taken
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int e = lane + 32 * k;
        key[k] = (e < experts) ? logit_key(s.logit[e]) : int(0x80000000u);
        live |= (e < experts) ? (1u << k) : 0u;
    }
#pragma unroll
    for (int r = 0; r < kTopK; ++r) {
        // this lane's best expert in play: the largest key, the lowest k among equal keys
        int best = int(0x80000000u);
        int bk = -1;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (((live >> k) & 1u) && (bk < 0 || key[k] > best)) {
                best = key[k];
                bk = k;
            }
        }
        const int m = __reduce_max_sync(0xffffffffu, best);
        const unsigned cand = (bk >= 0 && best == m) ? unsigned(lane + 32 * bk) : 0xffffffffu;
        const unsigned win = __reduce_min_sync(0xffffffffu, cand);
        if (lane == 0) {
            s.sel[r] = (win < unsigned(experts)) ? int(win) : 0;
        }
        if (bk >= 0 && cand == win) {
            live &= ~(1u << bk);
        }
    }
}

// After warp_top4 and a compute_sync: whether a selected logit is NaN or a
// selected and another expert's logits are closer than their bounds (the f32
// order of the reference may differ); sets s.amb, which the caller zeroed
// before the last compute_sync.
__device__ __forceinline__ void check_top4(Smem &s, int experts) {
    bool amb = false;
    for (int e = threadIdx.x; e < experts; e += kComputeThreads) {
#pragma unroll
        for (int q = 0; q < kTopK; ++q) {
            const int a = s.sel[q];
            const float la = s.logit[a];
            amb = amb | !(la == la) | ((a != e) & !(fabsf(la - s.logit[e]) > s.bound[a] + s.bound[e]));
        }
    }
    if (amb) {
        s.amb = 1;
    }
}

// B-operand scales of one operand's chunks (kCols / 4 of them) into tensor
// memory: chunk c at columns 4c..4c+3, of which the MMA reads column 4c (lane
// n = row n of B, byte k = K-block 4c + k); four chunks per store.
// Warp-collective, this warp's lane quadrant.
template <uint32_t kCols = kSfbCols>
__device__ __forceinline__ void store_sfb(const uint8_t *codes, uint32_t taddr, int lane) {
    static_assert(kCols % 16 == 0, "whole stores");
#pragma unroll
    for (int g4 = 0; g4 < int(kCols / 16); ++g4) {
        uint32_t v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            v[k] = (k & 3) ? 0u
                           : tc::digit_scales4(*reinterpret_cast<const uint32_t *>(codes + 16 * g4 + (k & ~3)), lane);
        }
        tc::tmem_st16(taddr + 16 * uint32_t(g4), v);
    }
    tc::wait_st();
}

// Softmax of the selected logits (src/model.cpp:310-321) and this rank's
// experts, by warp 0 (lane q handles selection q; the maximum and the sum
// run in rank order as in the reference), then published to the load warp.
// Called by all 32 lanes of warp 0 after s.sel is visible to them.
__device__ __forceinline__ void publish_selection(Smem &s, const StackArgs &a, bool export_top, int step) {
    const int lane = threadIdx.x & 31;
    const int q = lane & 3;
    const int e = s.sel[q];
    const float v = s.val[e];
    float v4[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        v4[k] = __shfl_sync(0xffffffffu, v, k);
    }
    float maximum = -INFINITY;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        maximum = (maximum < v4[k]) ? v4[k] : maximum;
    }
    const float wq = expf(__fsub_rn(v, maximum));
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
        sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, wq, k));
    }
    const int le = e - a.expert_begin;
    const bool mine = (le >= 0) & (le < a.expert_count) & (lane < kTopK);
    const unsigned owned = __ballot_sync(0xffffffffu, mine);
    if (lane < kTopK) {
        s.wts[q] = __fdiv_rn(wq, sum);
        s.local[q] = mine ? le : -1;
        if (mine) {
            s.slot_of[__popc(owned & ((1u << lane) - 1u))] = q;
        }
        if (export_top) {
            a.top_idx[q] = e;
            a.top_w[q] = __fdiv_rn(wq, sum);
            if (a.mode == 2) {  // the server's top-4, tagged with the request's number
                const uint32_t r = a.mbox_base + uint32_t(step) + 1u;
                const unsigned long long wi = (static_cast<unsigned long long>(r) << 32) | uint32_t(e);
                asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a.mbox->top + q), "l"(wi) : "memory");
                asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a.mbox->top + 4 + q),
                             "l"(tagged(r, __fdiv_rn(wq, sum)))
                             : "memory");
            }
        }
        if (a.ilog && blockIdx.x == 0 && step < a.log_steps) {
            a.ilog[size_t(step) * kTopK + q] = e;
            a.wlog[size_t(step) * kTopK + q] = __fdiv_rn(wq, sum);
        }
    }
    if (lane == 0) {
        s.n_local = __popc(owned);
    }
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(&s.sel_full);
    }
}

// Load warp: every step's stages, following the published selections; at the
// end it waits until every load it issued has landed.
// ---- the decode server (mode 2) ----
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The layer of step `step`'s request, on every compute thread of every CTA,
// or -1 when the server leaves.  CTA 0 polls the mailbox in host memory
// (bounded by the idle limit, or until the host asks it to stop), copies the
// request's x into device memory and publishes (step tag, layer) in a.go;
// the other CTAs poll that word (bounded by the idle limit + 2 s).
__device__ int server_next(Smem &s, const StackArgs &a, int step) {
    const int ct = threadIdx.x;
    const uint32_t tag = step_tag(s, step);
    if (blockIdx.x == 0) {
        if (ct == 0) {
            int layer = -1;
            const uint32_t want = a.mbox_base + uint32_t(step) + 1u;
            const unsigned long long t0 = tc::now_ns();
            for (;;) {
                unsigned long long w;
                asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(&a.mbox->reqw) : "memory");
                if (uint32_t(w >> 32) == want) {
                    layer = int(uint32_t(w));
                    if (layer < a.layer_begin || layer >= a.layer_end) {
                        set_status(a.status, kStatusBadShape);  // the host checks the layer first
                        layer = -1;
                    }
                    break;
                }
                if (ld_acquire_sys(&a.mbox->stop) != 0u || tc::now_ns() - t0 > a.idle_ns) {
                    break;
                }
            }
            if (layer < 0) {
                st_release_sys(&a.mbox->alive, 0u);  // no request is taken after this
            }
            s.srv_layer = layer;
        }
        compute_sync();
        if (s.srv_layer >= 0) {
            // 720 float4 over PCIe: each thread's loads all in flight, then stored
            constexpr int kVec = kDim / 4;
            constexpr int kPer = (kVec + kComputeThreads - 1) / kComputeThreads;  // 3
            const float4 *__restrict__ src = reinterpret_cast<const float4 *>(a.mbox->x);
            float4 *__restrict__ dst = reinterpret_cast<float4 *>(a.srv_x);
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int k = ct + j * kComputeThreads;
                if (k < kVec) {
                    dst[k] = __ldcv(src + k);
                }
            }
            __threadfence();
        }
        compute_sync();
        if (ct == 0) {
            const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | uint32_t(s.srv_layer);
            asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(a.go), "l"(w) : "memory");
        }
    } else {
        if (ct == 0) {
            int layer = -1;
            const unsigned long long t0 = tc::now_ns();
            for (;;) {
                unsigned long long w;
                asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(a.go) : "memory");
                if (uint32_t(w >> 32) == tag) {
                    layer = int(uint32_t(w));
                    break;
                }
                if (tc::now_ns() - t0 > a.idle_ns + kGridWaitNs) {
                    fail_wait(s, a.status);
                    break;
                }
            }
            s.srv_layer = layer;
        }
        compute_sync();
    }
    if (ct == 0) {
        s.step_layer = s.srv_layer;
    }
    compute_sync();
    return s.srv_layer;
}

// CTA 0 reports a step that failed: when the device status word is set at
// the step's end, it goes to the mailbox with the request's number in `resp`
// (the host then stops the server and reads the status).  A step that went
// well needs nothing here: its rows and top-4 are tagged words.
__device__ void server_answer(Smem &s, const StackArgs &a, int step) {
    if (blockIdx.x != 0 || threadIdx.x != 0) {
        return;
    }
    const uint32_t st = *reinterpret_cast<const volatile uint32_t *>(a.status);
    if (st) {
        a.mbox->status = st;
        __threadfence_system();
        st_release_sys(&a.mbox->resp, a.mbox_base + uint32_t(step) + 1u);
    }
}

__device__ void run_loads(const Ctx &c0, Smem &s, const StackArgs &a, int steps, int nl) {
    Pipe pp;
    for (int step = 0; step < steps; ++step) {
        if (!wait_bar(s, &s.sel_full, uint32_t(step) & 1, a.status)) {
            break;
        }
        if (a.mode == 2 && *reinterpret_cast<const volatile int *>(&s.srv_exit)) {
            break;  // the server took no further request
        }
        int le[kTopK];
        const int n = s.n_local;
#pragma unroll
        for (int q = 0; q < kTopK; ++q) {
            le[q] = (q < n) ? s.local[s.slot_of[q]] : 0;
        }
        Ctx c = c0;
        c.L = &a.layers[a.mode == 2 ? s.step_layer : a.layer_begin + step % nl];
        if (!produce_phase(c, s.plan[n][0], 0, le, pp) || !produce_phase(c, s.plan[n][1], 1, le, pp)) {
            break;
        }
        // the next step's tensor maps, while this step's loads are in flight
        if (a.mode != 2 && step + 1 < steps) {
            const TmaDesc *nt = a.layers[a.layer_begin + (step + 1) % nl].tma;
#pragma unroll
            for (int m = 0; m < kTmaCount; ++m) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(nt + m) : "memory");
            }
        }
    }
    for (uint32_t k = 0; k < kStages && k < pp.stage; ++k) {
        const uint32_t last = pp.stage - 1 - k;
        tc::mbar_wait(&s.full[last % kStages], (last / kStages) & 1);
    }
}

// kWideRouter: more experts than kPreE (gpt-oss-120b), whose next-layer router
// weights the down reducers stage through shared memory; a separate
// instantiation, so the 32-expert kernel carries none of it.
template <bool kWideRouter>
__global__ void __launch_bounds__(kThreads, 1) decode_tc_kernel(StackArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // aligned by offsetting the shared array itself, so that accesses through
    // s stay shared-memory accesses (a detour through an integer address
    // would make every one of them a generic access)
    Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int E = a.experts;
    const int nl = steps_per_token(a);
    const int steps = a.tokens * nl;
    unsigned gen = 0;

    if (threadIdx.x == 0) {
        s.abort = 0;
        s.srv_exit = 0;
        s.steps_run = uint32_t(steps);
        // the tag base lives on the device, so a replayed graph of this launch
        // gets new tags: the last CTA to finish advances it by the steps
        s.seq = *reinterpret_cast<const volatile uint32_t *>(a.seq_state);
        for (int i = 0; i < kStages; ++i) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], kIssuers);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&s.acc_full[i], kIssuers);
            tc::mbar_init(&s.acc_empty[i], 32 * kEpiWarps);
        }
        tc::mbar_init(&s.sel_full, 1);
        tc::mbar_init(&s.setup, 1);
        tc::mbar_init(&s.rwbar, 1);
        s.rw_uses = 0;
        s.rw_issued = 0;
        tc::mbar_init(&s.fin, kIssuers);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&s.tmem, kTmemCols);
        tc::tmem_relinquish();
    }
    // padding of the gate/up block codes (K-blocks 90..95)
    if (threadIdx.x < kCodeBytes - kBlocks) {
        s.gcode[kBlocks + threadIdx.x] = 127u;
    }
    // work plans for 0..4 local experts: lane 0 of warp w builds (w / 2, w % 2)
    if (lane == 0 && warp < 2 * (kTopK + 1)) {
        const int n = warp >> 1;
        build_plan(s.plan[n][warp & 1], (warp & 1) ? down_phase(n) : gateup_phase(n), a.status);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before_sync();
    __syncwarp();  // warps reconverge before the block barrier (see compute_sync)
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = s.tmem;
    const Ctx c0{&a, &a.layers[a.layer_begin], &s, tbase};

    if (warp == kTmaWarp) {
        if (lane == 0) {
            run_loads(c0, s, a, steps, nl);
        }
    } else {
        // ---------------- compute group: warps 0-8 ----------------
        const int ct = threadIdx.x;  // 0..287
        Pipe pipe;
        unsigned want_b0 = 0, want_b1 = 0, want_b2 = 0, want_b3 = 0;  // warp 8, lane 0
        // Router sums of (token 0, first layer) in stack mode.
        if (a.mode == 1) {
            const StackLayer &L = a.layers[a.layer_begin];
            const int r0 = range_lo(blockIdx.x, gridDim.x, kDim);
            const int r1 = range_lo(blockIdx.x + 1, gridDim.x, kDim);
            for (int e = warp; e < E + 1; e += kComputeWarps) {
                double v = 0.0;
                for (int r = r0 + lane; r < r1; r += 32) {
                    const float xr = a.x[r];
                    v += (e < E) ? double(__ldg(L.router_w + size_t(e) * kDim + r)) * double(__fmul_rn(xr, L.norm_w[r]))
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
                const int step = t * nl + li;
                int l = a.layer_begin + li;
                if (a.mode == 2) {
                    // the server: the next request's layer (x is in a.srv_x), or leave
                    l = server_next(s, a, step);
                    if (l < 0) {
                        if (threadIdx.x == 0) {
                            s.steps_run = uint32_t(step) + 1u;  // the exit word used this step's tag
                            s.srv_exit = 1;
                            mbar_arrive(&s.sel_full);  // the loads warp sees the exit
                        }
                        ok = false;
                        break;
                    }
                }
                const StackLayer &L = a.layers[l];
                const int tr = t & a.row_mask;
                const float *xcur = (a.mode == 2) ? a.srv_x
                                    : (li == 0)   ? a.x + size_t(tr) * kDim
                                                  : a.y + size_t(tr) * kDim;
                const bool export_top =
                    blockIdx.x == 0 && (a.mode == 2 || (t == a.tokens - 1 && li == nl - 1));

                stamp(a, step, 0);
                // The gate/up B operand: digit terms of x * g (mode 1) or of h
                // (mode 0).  From the second step of a stack on, the previous
                // step's down epilogues have written it (a.bnext): one bulk
                // copy.  Otherwise it is split here from x (and g) staged in
                // shared memory by asynchronous copies issued now, before the
                // selection (the down-operand area is idle in such a step);
                // the split loop is not unrolled: it runs once per launch, so
                // its code is fetched cold, and unrolled it would miss the
                // instruction cache once per pass.
                const bool split_here = (a.mode != 1) || (step == 0);
                constexpr int kPasses = kBlocks / kComputeWarps;  // 10
                static_assert(kPasses * kComputeWarps == kBlocks, "split passes");
                static_assert(sizeof(Smem::bdown) >= 2 * kDim * sizeof(float), "split staging");
                float *xs = reinterpret_cast<float *>(&s.bdown[0][0][0]);
                float *gs = xs + kDim;
                if (split_here && a.mode == 2) {
                    // the server's input changes per request: read through L2
#pragma unroll 1
                    for (int k = ct; k < kDim; k += kComputeThreads) {
                        xs[k] = __ldcg(xcur + k);
                    }
                } else if (split_here) {
#pragma unroll 1
                    for (int k = ct; k < kDim; k += kComputeThreads) {
                        cp_async4(xs + k, xcur + k);
                        if (a.mode == 1) {
                            cp_async4(gs + k, L.norm_w + k);
                        }
                    }
                    asm volatile("cp.async.commit_group;" ::: "memory");
                }
                float scale = 1.0f;
                // ---------------- A: selection ----------------
                if (a.mode == 1) {
                    // the router bias is loaded before the wait for the sums
                    static_assert(kMaxExperts <= kComputeThreads, "one expert per compute thread");
                    const float rb = (ct < E) ? __ldg(L.router_b + ct) : 0.0f;
                    // router sums: the kernel's opening pass (step 0) or the
                    // previous step's down reducers
                    if (step > 0) {
                        static_assert(kTiles * (kPreE + 1) <= kComputeThreads * 3 &&
                                          kTiles * (kMaxExperts + 1) <= kComputeThreads * 11,
                                      "router sums in one round of polls");
                        gather_router_sums<kWideRouter ? 11 : 3>(s, a, step, E);
                    }
                    compute_sync();
                    stamp(a, step, 4);
                    const double *sums = (step > 0) ? &s.rsum[0][0] : a.acc;
                    const float ss = float(sums[E]);
                    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(kDim)), 1.0e-5f)));
                    if (ct < E) {
                        const float lg = float(double(rb) + double(scale) * sums[ct]);
                        s.logit[ct] = lg;
                        s.val[ct] = lg;
                    }
                    compute_sync();
                    if (warp == 0) {
                        warp_top4(s, E);
                        __syncwarp();
                        publish_selection(s, a, export_top, step);
                    }
                } else {
                    // CTA e < E: expert e's logit and the bound on the reference's f32 chain.
                    for (int e = blockIdx.x; e < E; e += gridDim.x) {
                        const float *wr = L.router_w + size_t(e) * kDim;
                        constexpr int kCols = kDim / kComputeWarps;  // 320 per warp
                        constexpr int kPer = (kCols + 31) / 32;      // 10 per lane
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
                        compute_sync();
                        if (lane == 31) {
                            s.red[warp] = inc;
                        }
                        compute_sync();
                        double base = double(L.router_b[e]);
                        double total = 0.0;
                        for (int k = 0; k < kComputeWarps; ++k) {
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
                        compute_sync();
                        if (lane == 0) {
                            s.red[warp] = abs_sum;
                        }
                        compute_sync();
                        if (threadIdx.x == 0) {
                            double abs_total = 0.0;
                            for (int k = 0; k < kComputeWarps; ++k) {
                                abs_total += s.red[k];
                            }
                            const double logit = double(L.router_b[e]) + total;
                            const float bound = float((1.02 * 5.9604644775390625e-08 * abs_total +
                                                       5.9604644775390625e-08 * fabs(logit) + 1e-30) *
                                                      1.0001);
                            // (logit, bound) as two tagged words in one 16-byte store
                            asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(
                                             a.rlog + (size_t(step & 1) * kMaxExperts + size_t(e)) * 2),
                                         "l"(tagged(step_tag(s, step), float(logit))), "l"(tagged(step_tag(s, step), bound))
                                         : "memory");
                        }
                        compute_sync();
                    }
                    // every expert's (logit, bound) pair, polled as soon as its CTA
                    // stored it (no grid barrier: a CTA cannot be two steps ahead of
                    // another, since each step's reductions need every CTA's partials)
                    static_assert(kMaxExperts <= kComputeThreads, "one expert per compute thread");
                    if (ct < E) {
                        float lv[2] = {0.0f, 0.0f};
                        poll_tagged<2>(
                            s, [&](int k) { return a.rlog + (size_t(step & 1) * kMaxExperts + size_t(ct)) * 2 + k; },
                            3u, step_tag(s, step), lv, a.status);
                        s.logit[ct] = lv[0];
                        s.bound[ct] = lv[1];
                        s.val[ct] = lv[0];
                    }
                    compute_sync();
                    if (threadIdx.x == 0) {
                        s.amb = 0;
                        s.go = aborted(s) ? 0 : 1;
                    }
                    compute_sync();
                    ok = s.go != 0;
                    if (!ok) {
                        break;
                    }
                    if (warp == 0) {
                        warp_top4(s, E);
                    }
                    compute_sync();
                    check_top4(s, E);
                    compute_sync();
                    if (s.amb) {
                        float lower = INFINITY;
                        for (int q = 0; q < kTopK; ++q) {
                            lower = fminf(lower, s.logit[s.sel[q]] - s.bound[s.sel[q]]);
                        }
                        for (int e = ct; e < E; e += kComputeThreads) {
                            if (!(s.logit[e] + s.bound[e] < lower)) {
                                s.val[e] = exact_logit(L.router_w + size_t(e) * kDim, L.router_b[e], xcur);
                            }
                        }
                        compute_sync();
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
                        compute_sync();
                    }
                    if (warp == 0) {
                        publish_selection(s, a, export_top, step);
                    }
                }
                stamp(a, step, 1);
                if (threadIdx.x == 0) {
                    s.nscale = scale;
                }
                if (split_here) {
                    asm volatile("cp.async.wait_all;" ::: "memory");
                    compute_sync();
#pragma unroll 1
                    for (int pi = 0; pi < kPasses; ++pi) {
                        const int kb = warp + pi * kComputeWarps;
                        const int k = kb * 32 + lane;
                        const float h = (a.mode == 1) ? __fmul_rn(xs[k], gs[k]) : xs[k];
                        const uint32_t code = tc::digit_split_store(h, &s.bgu[kb][0], lane);
                        if (lane == 0) {
                            s.gcode[kb] = uint8_t(code);
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                } else {
                    gather_next_operand(s, a, step);
                }
                compute_sync();
                if (warp < kEpiWarps) {
                    store_sfb(s.gcode, tbase + (uint32_t(32 * warp) << 16) + kColSfbG, lane);
                }
                tc::fence_before_sync();
                compute_sync();
                tc::fence_after_sync();

                stamp(a, step, 2);
                // ---------------- B: gate/up ----------------
                Ctx cx{&a, &L, &s, tbase};
                const Phase pb = gateup_phase(s.n_local);
                const Plan &plb = s.plan[s.n_local][0];
                if (warp < kEpiWarps) {
                    run_epilogue<kWideRouter>(cx, pb, plb, pipe, t, li, false);
                } else if (warp < kIssuerWarp0 + kIssuers && lane == 0) {
                    run_mma(cx, plb, 0, pipe, warp - kIssuerWarp0);
                }
                __syncwarp();
                stamp(a, step, 3);
                // ---------------- C: down ----------------
                // B for down: the w * hidden terms (written by phase B's reducers)
                // of the experts this CTA's down units touch (at most kDownSlots),
                // into shared memory; their scales into tensor memory.
                if (warp == kMmaWarp && lane == 0) {
                    // bdown slots of the experts this CTA's down units touch
                    // (at most kDownSlots), fetched by bulk copies
                    const Plan &pd = s.plan[s.n_local][1];
                    for (int q = 0; q < kTopK; ++q) {
                        s.dslot[q] = -1;
                    }
                    // gate/up tiles each expert slot has had reduced through this step
                    const int nloc = s.n_local;
                    want_b0 += (nloc > 0) ? unsigned(kTiles) : 0u;
                    want_b1 += (nloc > 1) ? unsigned(kTiles) : 0u;
                    want_b2 += (nloc > 2) ? unsigned(kTiles) : 0u;
                    want_b3 += (nloc > 3) ? unsigned(kTiles) : 0u;
                    static_assert(kDownSlots == 2, "two down slots");
                    int qs0 = 0, qs1 = 0;
                    int nd = 0;
                    for (int si = 0; si < pd.nst; ++si) {
                        const int q = pd.st[si].q;
                        if (s.dslot[q] < 0) {
                            if (nd < kDownSlots) {
                                if (nd == 0) {
                                    qs0 = q;
                                } else {
                                    qs1 = q;
                                }
                                s.dslot[q] = nd++;
                            } else {
                                set_status(a.status, kStatusBadShape);
                                s.dslot[q] = 0;
                            }
                        }
                    }
                    // the down B operand of these slots is complete once all their
                    // gate/up tiles of this step are reduced
                    for (int d = 0; d < nd; ++d) {
                        const int q = (d == 0) ? qs0 : qs1;
                        const unsigned want = (q == 0) ? want_b0 : (q == 1) ? want_b1 : (q == 2) ? want_b2 : want_b3;
                        wait_count(s, a.cnt_b + q, want, a.status);
                    }
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc::mbar_expect_tx(&s.setup, uint32_t(nd) * uint32_t(kBlocks * kBRowBytes + kCodeBytes));
                    const uint8_t *bd = a.bdown + size_t(step & 1) * (kBdownBytes / 2);
                    const uint8_t *sd = a.sfb_down + size_t(step & 1) * (kSfbDownBytes / 2);
                    for (int d = 0; d < nd; ++d) {
                        const int q = (d == 0) ? qs0 : qs1;
                        bulk_load(&s.bdown[d][0][0], bd + size_t(q) * kBlocks * kBRowBytes, kBlocks * kBRowBytes, &s.setup);
                        bulk_load(&s.dcode[d][0], sd + size_t(q) * kCodeBytes, kCodeBytes, &s.setup);
                    }
                }
                if (warp < kEpiWarps && lane == 0 && !wait_bar(s, &s.setup, uint32_t(step) & 1, a.status)) {
                    *reinterpret_cast<volatile int *>(&s.abort) = 1;
                }
                __syncwarp();
                compute_sync();
                // slot d's scales by warps 4d .. 4d + 3 (warp w reaches lanes 32 (w % 4) ..)
                static_assert(kDownSlots * 4 <= kComputeWarps, "one warp quadrant set per down slot");
                if (warp < 4 * kDownSlots) {
                    const int d = warp >> 2;
                    store_sfb(s.dcode[d], tbase + (uint32_t(32 * (warp & 3)) << 16) + kColSfbD + kSfbCols * d, lane);
                }
                tc::fence_before_sync();
                compute_sync();
                tc::fence_after_sync();
                stamp(a, step, 5);
                const bool next_router = (a.mode == 1) && (li + 1 < nl || t + 1 < a.tokens);
                const Phase pc = down_phase(s.n_local);
                const Plan &plc = s.plan[s.n_local][1];
                if (warp < kEpiWarps) {
                    run_epilogue<kWideRouter>(cx, pc, plc, pipe, t, li, next_router);
                } else if (warp < kIssuerWarp0 + kIssuers && lane == 0) {
                    run_mma(cx, plc, 1, pipe, warp - kIssuerWarp0);
                }
                __syncwarp();
                stamp(a, step, 6);
                // every compute thread leaves or stays together
                compute_sync();
                if (a.mode == 2) {
                    server_answer(s, a, step);
                }
                if (threadIdx.x == 0) {
                    s.go = aborted(s) ? 0 : 1;
                }
                compute_sync();
                ok = s.go != 0;
                stamp(a, step, 7);
            }
        }
        if (!ok) {
            *reinterpret_cast<volatile int *>(&s.abort) = 1;
        }
        // the MMA issuers wait for their MMAs
        if (warp >= kIssuerWarp0 && warp < kIssuerWarp0 + kIssuers && lane == 0) {
            tc::mma_commit(&s.fin);
            tc::mbar_wait(&s.fin, 0);
        }
        // a router-weight staging whose wait gave up (the launch is aborting)
        // still has its copies in flight: wait for them once more (bounded)
        // before the shared memory is released
        if (kWideRouter && threadIdx.x == 0 && s.rw_issued != s.rw_uses) {
            if (!tc::mbar_wait(&s.rwbar, s.rw_uses & 1u)) {
                set_status(a.status, kStatusWaitTimeout);
            }
        }
    }
    tc::fence_before_sync();
    __syncwarp();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kTmemCols);
    }
    if (a.mode == 2 && blockIdx.x == 0 && threadIdx.x == 0) {
        st_release_sys(&a.mbox->alive, 0u);  // however the server ends, it takes no more requests
    }
    if (threadIdx.x == 0) {
        unsigned done;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(done) : "l"(a.seq_state + 1) : "memory");
        if (done == gridDim.x - 1) {
            a.seq_state[0] = s.seq + s.steps_run;
            a.seq_state[1] = 0u;
        }
    }
}

} // namespace

size_t decode_tc_smem_bytes() {
    return sizeof(Smem) + 1024;
}

void configure_decode_tc() {
    cudaFuncSetAttribute(decode_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(decode_tc_smem_bytes()));
    cudaFuncSetAttribute(decode_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(decode_tc_smem_bytes()));
}

cudaError_t launch_decode_tc(const StackArgs &args, int sms, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = decode_tc_smem_bytes();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return args.experts > kPreE ? cudaLaunchKernelEx(&cfg, decode_tc_kernel<true>, args)
                                : cudaLaunchKernelEx(&cfg, decode_tc_kernel<false>, args);
}

} // namespace ttl
