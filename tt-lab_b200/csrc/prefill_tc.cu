// prefill_tc.cu -- the expert products of a batched (prefill) MoE on the
// tcgen05 tensor cores.
//
// Reference: GptOssModel::moe_batch, tt-lab src/model.cpp:396-448 (the
// per-expert gate/up matmul with SwiGLU, :423-433, and the down matmul).
//
// Work is grouped by expert: prefill.cu's routing pads each local expert's
// routed pairs to a multiple of 16 slots, and a group is 16 slots of one
// expert.  Products are kind::mxf4 block-scaled MMAs, M = 128 weight rows,
// N = 128, K = 64: A is the expert's packed E2M1 weights with their own E8M0
// scales (the decode kernel's tensor maps and scale blocks, untouched), B is
// the group's activations in block fixed point -- per slot and 32-value
// K-block, eight base-4 digit rows (E2M1 values 0..3) of the 16-bit mantissa
// |v| * 2^(15 - e), row d scaled by 2^(e - 15 + 2d), e the exponent of the
// block's largest |v| -- so 16 slots x 8 digits fill N = 128.  The digits
// are exact to 2^-16 of each K-block's largest value; the epilogue adds a
// slot's 8 digit columns.
//
//   prefill_split_kernel   one CTA per group: the B rows of the group (x of
//                          each slot's token) and their scale blocks, written
//                          once.
//   prefill_mma_kernel<1>  gate/up, persistent: item = (128-row tile, group);
//                          two MMA issuers (gate, up) into two accumulators;
//                          the epilogue applies the biases and SwiGLU, and
//                          each of its warps -- 32 rows of the tile, which are
//                          one K-block of the down product -- splits its
//                          slots' values into the down B operand directly.
//   prefill_mma_kernel<0>  down, persistent: item = (128-row tile, pair of
//                          consecutive groups of one expert); the stage's
//                          weight box is shared, issuer m multiplies it by
//                          group m's B rows into accumulator m; the epilogue
//                          adds the bias.
// Items run row-tile-major, so the groups of one expert read the same weight
// tile at about the same time (from L2 after the first).
// Every wait is bounded; on timeout the kernels record kStatusWaitTimeout.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace ttl {
namespace {

constexpr int kGroup = 16;                        // slots per group
constexpr int kDigits = 8;                        // digit rows per slot
constexpr int kPadBlocks = 96;                    // K-blocks per B row (90 + zero padding)
constexpr int kGroupKbBytes = kGroup * kDigits * 16;  // 2048: one K-block of a group's B rows
constexpr int kBoxes = 12;                        // 8-K-block weight boxes per row
constexpr int kStg = 4;                           // stage ring depth
constexpr int kEpiThreads = 128;                  // warps 0-3
constexpr int kProducerWarp = 4;
constexpr int kIssuerWarp0 = 5;                   // warps 5, 6
constexpr int kThreads = 32 * 7;
constexpr uint32_t kCols = 512;
constexpr uint32_t kColD = 0;                     // 2 x 128 accumulator columns
constexpr uint32_t kColSfa = 256;                 // kStg x 2 issuers x 2 chunks x 4 columns
constexpr uint32_t kColSfb = kColSfa + 16 * kStg; // same shape, each issuer its own copy
static_assert(kColSfb + 16 * kStg <= kCols, "tensor memory map");
static_assert(kGroupKbBytes * kPadBlocks == int(kPrefillGroupBytes), "group layout");
static_assert(24 * kScaleBlockBytes == int(kPrefillGroupScaleBytes), "group scale layout");

// Scale bytes of digit row d for four K-blocks' codes (one per byte): the
// E8M0 of 2^(e - 15 + 2d) is code - (15 - 2d); NaN codes stay NaN.
__device__ __forceinline__ uint32_t digit_scales8(uint32_t codes4, int d) {
    const uint32_t v = __vsubus4(codes4, uint32_t(15 - 2 * d) * 0x01010101u);
    const uint32_t nan = __vcmpeq4(codes4, 0xFFFFFFFFu);
    return (v & ~nan) | nan;
}

// Splits one K-block (warp-collective, one value per lane) into eight digit
// rows and writes them to `dst` ([8 rows][16 B], the MMA's core-matrix
// order).  Returns the block code e + 127 (127 for an all-zero block, 255 for
// inf or NaN).
__device__ __forceinline__ uint32_t digit_split8_store(float v, uint8_t *dst, int lane) {
    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    uint32_t code, m = 0u;
    if (mb >= 0x7f800000u) {
        code = 255u;
    } else if (mb == 0u || int(mb >> 23) < 27) {  // zero, or every |v| below 2^-100
        code = 127u;
    } else {
        const int e = int(mb >> 23) - 127;
        // |v| * 2^(15-e) < 2^16; truncated so the top digit stays below 4
        m = __float2uint_rz(__fmul_rn(fabsf(v), __uint_as_float(uint32_t(142 - e) << 23)));
        code = uint32_t(e + 127);
    }
    const uint32_t neg = __float_as_uint(v) >> 31;
    const uint32_t rows = tc::transpose_nibbles(tc::digit_codes(tc::spread_digits(m), neg), lane);
    *reinterpret_cast<uint32_t *>(dst + (lane & 7) * 16 + 4 * (lane >> 3)) = rows;
    return code;
}

// One CTA per group: its B rows ([96 K-blocks][16 slots][8 rows][16 B]) and
// the scale blocks of its 24 chunks of 4 K-blocks (row m = slot * 8 + digit
// at [m % 32][m / 32][K-block % 4], the order tcgen05.cp 32x128b moves).
// Slot rows are x of the slot's token (zero for padding slots).
__global__ void __launch_bounds__(32 * kGroup) prefill_split_kernel(PrefillWork w, const float *__restrict__ x) {
    __shared__ uint8_t codes[kGroup][kPadBlocks];
    const int g = blockIdx.x;
    if (g >= *w.tile_count) {
        return;
    }
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int code = w.tiles[g];
    const int le = code >> 20;
    const int first = code & 0xfffff;
    const int nvalid = min(kGroup, w.offsets[le] + w.counts[le] - first);
    uint8_t *dst = w.bdig + size_t(g) * kPrefillGroupBytes;
    // warp w splits slot w's row (16 warps, 16 slots), eight K-blocks' loads in flight
    const int slot = warp;
    const float *row = nullptr;
    if (slot < nvalid) {
        row = x + size_t(w.pair_token[first + slot]) * kDim;
    }
    static_assert(kPadBlocks % 8 == 0, "K-blocks in batches of 8");
    for (int kb0 = 0; kb0 < kPadBlocks; kb0 += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[j] = (row && kb0 + j < kBlocks) ? __ldcg(row + (kb0 + j) * 32 + lane) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int kb = kb0 + j;
            const uint32_t c = digit_split8_store(v[j], dst + size_t(kb) * kGroupKbBytes + slot * kDigits * 16, lane);
            if (lane == 0) {
                codes[slot][kb] = uint8_t(c);
            }
        }
    }
    __syncthreads();
    uint32_t *sfb = reinterpret_cast<uint32_t *>(w.bsfb + size_t(g) * kPrefillGroupScaleBytes);
    for (int idx = threadIdx.x; idx < 24 * 128; idx += blockDim.x) {
        const int chunk = idx >> 7;
        const int m = idx & 127;
        const uint32_t codes4 = *reinterpret_cast<const uint32_t *>(&codes[m >> 3][4 * chunk]);
        sfb[chunk * 128 + (m & 31) * 4 + (m >> 5)] = digit_scales8(codes4, m & 7);
    }
}

// A stage holds three 16 KB operand tiles: gate/up -- the gate box, the up
// box (swizzled) and the group's B rows of the box's 8 K-blocks; down -- the
// down box and the B rows of the pair's two groups.
struct alignas(1024) PSmem {
    uint8_t t[kStg][3][16384];                    // operand tiles (weight boxes at 1024-byte boundaries)
    uint8_t sfa[kStg][2][2][kScaleBlockBytes];    // [box][chunk] weight scale blocks
    uint8_t sfb[kStg][2][2][kScaleBlockBytes];    // [group][chunk] B scale blocks
    uint64_t full[kStg];
    uint64_t empty[kStg];
    uint64_t acc_full;
    uint64_t acc_empty;
    uint64_t fin;
    uint32_t tmem;
    int go;
};
static_assert(sizeof(PSmem) + 1024 <= 232448, "shared memory per CTA");
static_assert(offsetof(PSmem, t) % 1024 == 0 && offsetof(PSmem, sfa) % 16 == 0 && offsetof(PSmem, sfb) % 16 == 0,
              "copy destinations");
static_assert(8 * kGroupKbBytes == 16384 && 128 * 128 == 16384, "operand tiles");

__device__ __forceinline__ void bulk(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ bool wait(uint64_t *bar, uint32_t parity, uint32_t *status) {
    if (tc::mbar_wait(bar, parity)) {
        return true;
    }
    set_status(status, kStatusWaitTimeout);
    return false;
}

// Item i of `items` (row tile mt, unit u), row-tile-major.  A unit is one
// group (gate/up) or an entry of the pair list (down): groups g .. g + n - 1.
struct Item {
    int mt, g, n, le;
};
template <bool kGateUp>
__device__ __forceinline__ Item item_of(const PrefillWork &w, int i, int units) {
    Item it;
    it.mt = i / units;
    const int u = i - it.mt * units;
    if (kGateUp) {
        it.g = u;
        it.n = 1;
    } else {
        const int code = w.dtiles[u];
        it.g = code & 0xffffff;
        it.n = (code >> 24) + 1;
    }
    it.le = w.tiles[it.g] >> 20;
    return it;
}

// First slot and valid slots of group g.
__device__ __forceinline__ int2 group_slots(const PrefillWork &w, int g) {
    const int code = w.tiles[g];
    const int le = code >> 20;
    const int first = code & 0xfffff;
    return make_int2(first, min(kGroup, w.offsets[le] + w.counts[le] - first));
}

// K-blocks of box x (8, or 2 for the last box).
__device__ __forceinline__ int box_blocks(int x) {
    return min(8, kBlocks - 8 * x);
}

__device__ __forceinline__ void arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

// Stage k of an item is weight box k (8 K-blocks) with the B rows and scale
// blocks of those K-blocks.  Gate/up: the stage holds box k of gate (tile 0)
// and of up (tile 1) and the group's B rows (tile 2); issuer 0 multiplies
// gate, issuer 1 up, each into its accumulator.  Down: the stage holds box k
// of down (tile 0) and the B rows of the pair's groups (tiles 1, 2); issuer m
// multiplies the box by group m into accumulator m (idle when the pair has
// one group).
template <bool kGateUp>
__global__ void __launch_bounds__(kThreads, 1) prefill_mma_kernel(LayerDev L, const TmaDesc *tma, PrefillWork w) {
    extern __shared__ __align__(1024) unsigned char raw[];
    PSmem &s = *reinterpret_cast<PSmem *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int units = kGateUp ? *w.tile_count : *w.dtile_count;
    const int items = kScaleTiles * units;
    constexpr int kBoxA = kGateUp ? 2 : 1;  // weight boxes per stage
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStg; ++i) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], 2);
        }
        tc::mbar_init(&s.acc_full, 2);
        tc::mbar_init(&s.acc_empty, kEpiThreads);
        tc::mbar_init(&s.fin, 2);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&s.tmem, kCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncwarp();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tbase = s.tmem;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            uint32_t stage = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && i < items; i += gridDim.x) {
                const Item it = item_of<kGateUp>(w, i, units);
                const uint8_t *bg = (kGateUp ? w.bdig : w.bdig_dn) + size_t(it.g) * kPrefillGroupBytes;
                const uint8_t *sg = (kGateUp ? w.bsfb : w.bsfb_dn) + size_t(it.g) * kPrefillGroupScaleBytes;
                for (int k = 0; k < kBoxes; ++k, ++stage) {
                    const uint32_t st = stage % kStg;
                    const uint32_t use = stage / kStg;
                    if (use > 0 && !(ok = wait(&s.empty[st], (use - 1) & 1, w.status))) {
                        break;
                    }
                    const int nchunk = (box_blocks(k) + 3) / 4;
                    // full boxes are counted even where they reach past the matrix (zero fill)
                    const uint32_t tx = uint32_t(kBoxA) * (128 * 128 + uint32_t(nchunk) * kScaleBlockBytes) +
                                        uint32_t(it.n) * (8 * kGroupKbBytes + 2 * kScaleBlockBytes);
                    tc::mbar_expect_tx(&s.full[st], tx);
                    for (int b = 0; b < kBoxA; ++b) {
                        const int map = kGateUp ? (b == 0 ? kTmaGate : kTmaUp) : kTmaDown;
                        const uint8_t *mat = kGateUp ? (b == 0 ? L.gate : L.up) : L.down;
                        tc::tma_load_3d(&s.t[st][b][0], tma + map, 128 * k, 128 * it.mt, it.le, &s.full[st]);
                        bulk(&s.sfa[st][b][0][0], mat + size_t(it.le) * kPackedMatrixBytes + scale_block_offset(it.mt, 2 * k),
                             uint32_t(nchunk) * kScaleBlockBytes, &s.full[st]);
                    }
                    for (int j = 0; j < it.n; ++j) {
                        bulk(&s.t[st][kBoxA + j][0], bg + size_t(j) * kPrefillGroupBytes + size_t(8 * k) * kGroupKbBytes,
                             8 * kGroupKbBytes, &s.full[st]);
                        bulk(&s.sfb[st][j][0][0],
                             sg + size_t(j) * kPrefillGroupScaleBytes + size_t(2 * k) * kScaleBlockBytes,
                             2 * kScaleBlockBytes, &s.full[st]);
                    }
                }
            }
            // every load issued has landed before the CTA exits
            for (uint32_t k = 0; k < kStg && k < stage; ++k) {
                const uint32_t last = stage - 1 - k;
                tc::mbar_wait(&s.full[last % kStg], (last / kStg) & 1);
            }
        }
    } else if (warp >= kIssuerWarp0 && warp < kIssuerWarp0 + 2) {
        if (lane == 0) {
            const int m = warp - kIssuerWarp0;
            const uint32_t t0 = tc::smem_u32(&s.t[0][0][0]);
            const uint32_t dcol = tbase + kColD + 128 * uint32_t(m);
            uint32_t stage = 0;
            uint32_t item_no = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && i < items; i += gridDim.x, ++item_no) {
                if (item_no > 0 && !(ok = wait(&s.acc_empty, (item_no - 1) & 1, w.status))) {
                    break;
                }
                tc::fence_after_sync();
                // down: issuer 1 idles (but still releases the stages) for a one-group pair
                const bool active = kGateUp || m < item_of<kGateUp>(w, i, units).n;
                bool first = true;
                for (int k = 0; k < kBoxes; ++k, ++stage) {
                    const uint32_t st = stage % kStg;
                    if (!(ok = wait(&s.full[st], (stage / kStg) & 1, w.status))) {
                        break;
                    }
                    tc::fence_after_sync();
                    if (!active) {
                        tc::mma_commit(&s.empty[st]);
                        continue;
                    }
                    const int box = kGateUp ? m : 0;
                    const int grp = kGateUp ? 0 : m;
                    const int nkb = box_blocks(k);
                    const int nchunk = (nkb + 3) / 4;
                    const uint32_t sfa_col = tbase + kColSfa + 16 * st + 8 * uint32_t(m);
                    const uint32_t sfb_col = tbase + kColSfb + 16 * st + 8 * uint32_t(m);
                    for (int j = 0; j < nchunk; ++j) {
                        tc::sf_copy(sfa_col + 4 * j, tc::smem_u32(&s.sfa[st][box][j][0]));
                        tc::sf_copy(sfb_col + 4 * j, tc::smem_u32(&s.sfb[st][grp][j][0]));
                    }
                    const uint32_t abase = t0 + st * uint32_t(sizeof(s.t[0])) + uint32_t(box) * 16384u;
                    const uint32_t bbase = t0 + st * uint32_t(sizeof(s.t[0])) + uint32_t(kBoxA + grp) * 16384u;
                    for (int p = 0; 2 * p < nkb; ++p) {
                        const uint32_t sel = uint32_t((2 * p) & 3);
                        const uint32_t j = uint32_t(p >> 1);
                        const uint64_t ad = tc::smem_desc_sw128(abase + 32u * uint32_t(p));
                        const uint64_t bd = tc::smem_desc(bbase + uint32_t(2 * p) * kGroupKbBytes, kGroupKbBytes, 128);
                        tc::mma_f4(dcol, ad, bd, tc::instr_desc_f4(128, sel), (sfa_col + 4 * j) | (sel << 30),
                                   (sfb_col + 4 * j) | (sel << 30), !first);
                        first = false;
                    }
                    tc::mma_commit(&s.empty[st]);
                }
                if (!ok) {
                    break;
                }
                tc::mma_commit(&s.acc_full);
            }
            // the issued MMAs complete before the tensor memory is freed
            tc::mma_commit(&s.fin);
            tc::mbar_wait(&s.fin, 0);
        }
    } else if (warp < 4) {
        // epilogue: thread i = row i of the tile (TMEM lane i)
        const int i = threadIdx.x;
        uint32_t item_no = 0;
        for (int ii = blockIdx.x; ii < items; ii += gridDim.x, ++item_no) {
            const Item it = item_of<kGateUp>(w, ii, units);
            const int2 gs0 = group_slots(w, it.g);
            const int row = 128 * it.mt + i;
            float bias0 = 0.0f, bias1 = 0.0f;
            if (row < kDim) {
                if (kGateUp) {
                    bias0 = __ldg(L.gate_b + size_t(it.le) * kDim + row);
                    bias1 = __ldg(L.up_b + size_t(it.le) * kDim + row);
                } else {
                    bias0 = __ldg(L.down_b + size_t(it.le) * kDim + row);
                }
            }
            if (i == 0) {
                s.go = wait(&s.acc_full, item_no & 1, w.status) ? 1 : 0;
            }
            __syncwarp();
            asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
            const bool go = s.go != 0;
            asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
            if (!go) {
                break;
            }
            tc::fence_after_sync();
            // each slot's 8 digit columns added up, four slots of both
            // accumulators per read; the accumulators are free once read
            const uint32_t lanebase = tbase + (uint32_t(32 * warp) << 16);
            float v0[kGroup], v1[kGroup];
#pragma unroll
            for (int c = 0; c < 128; c += 32) {
                float a0[16], a1[16], b0[16], b1[16];
                tc::tmem_ld16(lanebase + kColD + uint32_t(c), a0);
                tc::tmem_ld16(lanebase + kColD + uint32_t(c + 16), a1);
                tc::tmem_ld16(lanebase + kColD + 128 + uint32_t(c), b0);
                tc::tmem_ld16(lanebase + kColD + 128 + uint32_t(c + 16), b1);
                tc::wait_ld();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float g0 = 0.0f, g1 = 0.0f, u0 = 0.0f, u1 = 0.0f;
#pragma unroll
                    for (int d = 0; d < kDigits; ++d) {
                        g0 += a0[8 * h + d];
                        g1 += a1[8 * h + d];
                        u0 += b0[8 * h + d];
                        u1 += b1[8 * h + d];
                    }
                    v0[(c >> 3) + h] = g0;
                    v0[(c >> 3) + 2 + h] = g1;
                    v1[(c >> 3) + h] = u0;
                    v1[(c >> 3) + 2 + h] = u1;
                }
            }
            tc::fence_before_sync();
            arrive(&s.acc_empty);
            if (kGateUp) {
                // this warp's 32 rows are K-block 4 mt + warp of the down
                // product: each slot's 32 values become its 8 digit rows there
                // (zero for padding slots and rows past 2879), and lane j < 16
                // keeps slot j's block code for the scale bytes
                const int kb = 4 * it.mt + warp;
                uint8_t *dg = w.bdig_dn + size_t(it.g) * kPrefillGroupBytes + size_t(kb) * kGroupKbBytes;
                uint32_t mycode = 0;
#pragma unroll
                for (int slot = 0; slot < kGroup; ++slot) {
                    float h = 0.0f;
                    if (row < kDim && slot < gs0.y) {
                        h = swiglu_ref(__fadd_rn(bias0, v0[slot]), __fadd_rn(bias1, v1[slot]));
                    }
                    const uint32_t c = digit_split8_store(h, dg + slot * kDigits * 16, lane);
                    mycode = (lane == slot) ? c : mycode;
                }
                // digit row m = slot * 8 + d of chunk mt at [m % 32][m / 32][kb % 4]
                uint8_t *sf = w.bsfb_dn + size_t(it.g) * kPrefillGroupScaleBytes + size_t(it.mt) * kScaleBlockBytes;
#pragma unroll
                for (int q = lane; q < kGroup * kDigits; q += 32) {
                    const uint32_t c = __shfl_sync(0xffffffffu, mycode, q >> 3);
                    sf[(q & 31) * 16 + (q >> 5) * 4 + warp] = uint8_t(digit_scales8(c, q & 7));
                }
            } else if (row < kDim) {
                const int2 gs1 = it.n > 1 ? group_slots(w, it.g + 1) : make_int2(0, 0);
#pragma unroll
                for (int slot = 0; slot < kGroup; ++slot) {
                    if (slot < gs0.y) {
                        w.down[size_t(gs0.x + slot) * kDim + row] = __fadd_rn(bias0, v0[slot]);
                    }
                    if (slot < gs1.y) {
                        w.down[size_t(gs1.x + slot) * kDim + row] = __fadd_rn(bias0, v1[slot]);
                    }
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncwarp();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tbase, kCols);
    }
}

}  // namespace

void configure_prefill_tc() {
    cudaFuncSetAttribute(prefill_mma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(sizeof(PSmem) + 1024));
    cudaFuncSetAttribute(prefill_mma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(sizeof(PSmem) + 1024));
}

void launch_prefill_gateup(const LayerDev &L, const TmaDesc *tma, const PrefillWork &w, const PrefillShape &s,
                           const float *x, cudaStream_t stream) {
    const int groups = int(prefill_groups(size_t(s.tokens), size_t(s.expert_count)));
    prefill_split_kernel<<<groups, 512, 0, stream>>>(w, x);
    prefill_mma_kernel<true><<<s.sms, kThreads, sizeof(PSmem) + 1024, stream>>>(L, tma, w);
}

void launch_prefill_down(const LayerDev &L, const TmaDesc *tma, const PrefillWork &w, const PrefillShape &s,
                         cudaStream_t stream) {
    prefill_mma_kernel<false><<<s.sms, kThreads, sizeof(PSmem) + 1024, stream>>>(L, tma, w);
}

}  // namespace ttl
