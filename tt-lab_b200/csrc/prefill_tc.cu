// prefill_tc.cu -- the expert products of a batched (prefill) MoE on the
// tcgen05 tensor cores.
//
// Reference: GptOssModel::moe_batch, tt-lab src/model.cpp:396-448 (the
// per-expert gate/up matmul with SwiGLU, :423-433, and the down matmul).
//
// Work is grouped by expert: prefill.cu's routing pads each local expert's
// routed pairs to a multiple of 16 slots (a group), and a unit is one or two
// consecutive groups of one expert.  Products are kind::mxf4 block-scaled
// MMAs, M = 128 weight rows, K = 64, N = 96 per group: A is the expert's
// packed E2M1 weights with their own E8M0 scales (the decode kernel's tensor
// maps and scale blocks, untouched), B is the unit's activations in block
// fixed point -- per slot and 32-value K-block, the magnitude
// m = |v| * 2^(16 - e) rounded to the nearest integer (e the exponent of the
// block's largest |v|, so m <= 2^17) written as six balanced radix-8 digits, m = sum_d c_d 8^d with c_d in
// [-4, 4] (E2M1 values, the sign of v applied), digit row d scaled by
// 2^(e - 16 + 3d) -- so 16 slots x 6 digits fill N = 96 and a unit of two
// groups N = 192.  Each value is within 2^-17 of its K-block's largest |v|;
// the epilogue adds a slot's 6 digit columns.
//
//   prefill_split_kernel   one CTA per (unit, group, quarter of K): the B rows
//                          of its slots (x of each slot's token) and their
//                          scale bytes.
//   prefill_mma_kernel<1>  gate/up, persistent: item = (128-row tile, unit);
//                          two MMA issuers (gate, up) into two N <= 192
//                          accumulators; eight epilogue warps (four per group
//                          of the unit) apply the biases and SwiGLU, and each
//                          -- 32 rows of the tile, which are one K-block of
//                          the down product -- splits its slots' values into
//                          the down B operand.
//   prefill_mma_kernel<0>  down, persistent: item = (128-row tile, unit); two
//                          issuers take alternate stages into two
//                          accumulators; the epilogue adds them and the bias.
// Items run row-tile-major, so the units of one expert read the same weight
// tile at about the same time (from L2 after the first).
// Every wait is bounded; on timeout the kernels record kStatusWaitTimeout.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace ttl {
namespace {

constexpr int kGroup = 16;                        // slots per group
constexpr int kDigits = 6;                        // digit rows per slot
constexpr int kGroupRows = kGroup * kDigits;      // 96: N of one group
constexpr int kUnitRows = 2 * kGroupRows;         // 192: B rows of a unit
constexpr int kPadBlocks = 96;                    // K-blocks per B row (90 + zero padding)
constexpr int kUnitKbBytes = kUnitRows * 16;      // 3072: one K-block of a unit's B rows
constexpr int kBoxes = 12;                        // 8-K-block weight boxes per row
constexpr int kEpiThreads = 256;                  // warps 0-3 (group 0 of a unit) and 7-10 (group 1)
constexpr int kProducerWarp = 4;
constexpr int kIssuerWarp0 = 5;                   // warps 5, 6
constexpr int kEpiWarp1 = 7;
constexpr int kThreads = 32 * 11;
constexpr uint32_t kCols = 512;
constexpr uint32_t kColD = 0;                     // 2 x 192 accumulator columns
constexpr uint32_t kColSf = 2 * kUnitRows;        // [issuer][ring slot] 32 columns: A scales, then B scales at +8
static_assert(kColSf + 2 * 2 * 32 <= kCols, "tensor memory map");
static_assert(size_t(kUnitKbBytes) * kPadBlocks == kPrefillUnitBytes, "unit layout");
static_assert(size_t(24) * 2 * kScaleBlockBytes == kPrefillUnitScaleBytes, "unit scale layout");

// Scale bytes of digit row d for four K-blocks' codes (one per byte): the
// E8M0 of 2^(e - 16 + 3d) is code - (16 - 3d); NaN codes stay NaN.
__device__ __forceinline__ uint32_t digit_scales6(uint32_t codes4, int d) {
    const uint32_t v = __vsubus4(codes4, uint32_t(16 - 3 * d) * 0x01010101u);
    const uint32_t nan = __vcmpeq4(codes4, 0xFFFFFFFFu);
    return (v & ~nan) | nan;
}

// E2M1 codes of the six balanced radix-8 digits of m <= 2^17, digit d in
// nibble d (nibbles 6, 7 zero).  With m' = m + 4 * (1 + 8 + ... + 8^4) and o_d
// the octal digits of m', the digits are c_d = o_d - 4 (in [-4, 3]) for
// d < 5 and c_5 = o_5 (in [0, 4]), since m = sum_d c_d 8^d.  Magnitudes 0, 1,
// 2, 3, 4 are the E2M1 codes 0, 2, 4, 5, 6; the sign bit is
// sign(c) xor `negative`, on nonzero digits.  Per nibble, without branches.
__device__ __forceinline__ uint32_t radix8_codes(uint32_t m, uint32_t negative) {
    const uint32_t mp = m + 0x4924u;
    const uint32_t o = (mp & 0x7u) | ((mp << 1) & 0x70u) | ((mp << 2) & 0x700u) | ((mp << 3) & 0x7000u) |
                       ((mp << 4) & 0x70000u) | ((mp << 5) & 0x700000u);
    const uint32_t up = (o >> 2) & 0x11111u;                 // low five digits with o >= 4 (c >= 0)
    const uint32_t up_mask = up * 0xFu;
    const uint32_t a_up = o & 0x33333u;                      // o - 4
    const uint32_t a_down = ((~o) & 0x33333u) + 0x11111u;    // 4 - o
    const uint32_t a = (a_up & up_mask) | (a_down & ~up_mask & 0xFFFFFu) | (o & 0xF00000u);
    const uint32_t big = ((a + 0x111111u) >> 2) & 0x111111u; // |c| >= 3
    const uint32_t big_mask = big * 0xFu;
    const uint32_t code = ((a << 1) & ~big_mask) | ((a + 0x222222u) & big_mask);
    const uint32_t nonzero = (a | (a >> 1) | (a >> 2)) & 0x111111u;
    const uint32_t sign = ((~up & 0x11111u) ^ (0u - negative & 0x111111u)) & nonzero;
    return code | (sign << 3);
}

// Splits one K-block (warp-collective, one value per lane) into six digit
// rows and writes them to `dst` ([6 rows][16 B]: element k in byte k / 2,
// low nibble first -- the MMA's K-major order).  Returns the block code
// e + 127 (127 for an all-zero block, 255 for inf or NaN).
__device__ __forceinline__ uint32_t digit_split6_store(float v, uint8_t *dst, int lane) {
    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    uint32_t code, m = 0u;
    if (mb >= 0x7f800000u) {
        code = 255u;
    } else if (mb == 0u || int(mb >> 23) < 27) {  // zero, or every |v| below 2^-100
        code = 127u;
    } else {
        const int e = int(mb >> 23) - 127;
        // |v| * 2^(16-e) < 2^17 is exact in f32; rounded to nearest, m <= 2^17
        m = __float2uint_rn(__fmul_rn(fabsf(v), __uint_as_float(uint32_t(143 - e) << 23)));
        code = uint32_t(e + 127);
    }
    const uint32_t neg = __float_as_uint(v) >> 31;
    const uint32_t rows = tc::transpose_nibbles(radix8_codes(m, neg), lane);
    if ((lane & 7) < kDigits) {
        *reinterpret_cast<uint32_t *>(dst + (lane & 7) * 16 + 4 * (lane >> 3)) = rows;
    }
    return code;
}

// Unit code -> (first group, groups).
__device__ __forceinline__ int2 unit_groups(const PrefillWork &w, int u) {
    const int code = w.units[u];
    return make_int2(code & 0xffffff, (code >> 24) + 1);
}

// First slot and valid slots of group g.
__device__ __forceinline__ int2 group_slots(const PrefillWork &w, int g) {
    const int code = w.tiles[g];
    const int le = code >> 20;
    const int first = code & 0xfffff;
    return make_int2(first, min(kGroup, w.offsets[le] + w.counts[le] - first));
}

// Byte offset, in a unit's scale region, of digit row m's scale for K-block
// kb: chunk kb / 4, block m / 128, [m % 32][(m % 128) / 32][kb % 4].
__device__ __forceinline__ int unit_scale_offset(int m, int kb) {
    return (kb >> 2) * 1024 + (m >> 7) * 512 + (m & 31) * 16 + ((m >> 5) & 3) * 4 + (kb & 3);
}

// Item b = (unit, group j, quarter h of the K-blocks), warp w = slot w: the
// group's B rows of the unit ([96 K-blocks][192 rows][16 B], row =
// j * 96 + slot * 6 + digit; slots past the group's end are zero rows) for
// K-blocks 24 h .. 24 h + 23, and their scale bytes (6 of the unit's 24
// chunks).  A one-group unit's second group is left unwritten: its products
// use N = 96 and never read those rows.  The CTAs stride over the items of
// the routed units (the count is on the device), so the grid does not grow
// with the token capacity.
constexpr int kSplitBlocks = kPadBlocks / 4;  // K-blocks per split item
__global__ void __launch_bounds__(32 * kGroup) prefill_split_kernel(PrefillWork w, const float *__restrict__ x) {
    __shared__ __align__(4) uint8_t codes[kGroup][kSplitBlocks];
    const int items = 8 * *w.unit_count;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int slot = warp;
#pragma unroll 1
    for (int b = blockIdx.x; b < items; b += gridDim.x) {
        const int u = b >> 3;
        const int j = (b >> 2) & 1;
        const int kb_first = (b & 3) * kSplitBlocks;
        const int2 ug = unit_groups(w, u);
        if (j >= ug.y) {
            continue;  // uniform over the CTA
        }
        const int2 gs = group_slots(w, ug.x + j);
        const float *row = slot < gs.y ? x + size_t(w.pair_token[gs.x + slot]) * kDim : nullptr;
        uint8_t *dst = w.bdig + size_t(u) * kPrefillUnitBytes + (j * kGroupRows + slot * kDigits) * 16;
        static_assert(kSplitBlocks % 8 == 0, "K-blocks in batches of 8");
        for (int k0 = 0; k0 < kSplitBlocks; k0 += 8) {
            float v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int kb = kb_first + k0 + q;
                v[q] = (row && kb < kBlocks) ? __ldcg(row + kb * 32 + lane) : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int kb = kb_first + k0 + q;
                const uint32_t c = digit_split6_store(v[q], dst + size_t(kb) * kUnitKbBytes, lane);
                if (lane == 0) {
                    codes[slot][k0 + q] = uint8_t(c);
                }
            }
        }
        __syncthreads();
        // one word per (chunk, row): the row's scale bytes of the chunk's 4 K-blocks
        uint8_t *sfb = w.bsfb + size_t(u) * kPrefillUnitScaleBytes;
        for (int idx = threadIdx.x; idx < (kSplitBlocks / 4) * kGroupRows; idx += blockDim.x) {
            const int chunk = idx / kGroupRows;
            const int r = idx - chunk * kGroupRows;
            const int s = r / kDigits;
            *reinterpret_cast<uint32_t *>(sfb + unit_scale_offset(j * kGroupRows + r, kb_first + 4 * chunk)) =
                digit_scales6(*reinterpret_cast<const uint32_t *>(&codes[s][4 * chunk]), r - s * kDigits);
        }
        __syncthreads();  // codes is rewritten by the next item
    }
}

// Per-kernel shape: gate/up stages hold two weight boxes, down stages one.
template <bool kGateUp>
struct Cfg {
    static constexpr int kStg = kGateUp ? 3 : 5;  // stage ring depth
    static constexpr int kBoxA = kGateUp ? 2 : 1; // weight boxes per stage
};

// A stage: the weight box(es) of 8 K-blocks (swizzled, 1024-byte aligned),
// the unit's B rows of those K-blocks, and their scale blocks.
template <bool kGateUp>
struct alignas(1024) PSmem {
    static constexpr int kStg = Cfg<kGateUp>::kStg;
    static constexpr int kBoxA = Cfg<kGateUp>::kBoxA;
    uint8_t a[kStg][kBoxA][16384];
    uint8_t b[kStg][8 * kUnitKbBytes];
    uint8_t sfa[kStg][kBoxA][2][kScaleBlockBytes];  // [box][chunk]
    uint8_t sfb[kStg][2][2][kScaleBlockBytes];      // [chunk][block]
    uint64_t full[kStg];
    uint64_t empty[kStg];
    uint64_t sfree[2][2];   // [issuer][ring slot]: the slot's last MMAs have completed
    uint64_t acc_full;
    uint64_t acc_empty;
    uint64_t fin;
    uint32_t tmem;
    int go;
};
static_assert(sizeof(PSmem<true>) + 1024 <= 232448 && sizeof(PSmem<false>) + 1024 <= 232448,
              "shared memory per CTA");
static_assert(128 * 128 == 16384 && (8 * kUnitKbBytes) % 1024 == 0, "operand tiles");

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

// Item i of `items` (row tile mt, unit u), row-tile-major.
struct Item {
    int mt, u, g, n, le;
};
__device__ __forceinline__ Item item_of(const PrefillWork &w, int i, int units) {
    Item it;
    it.mt = i / units;
    it.u = i - it.mt * units;
    const int2 ug = unit_groups(w, it.u);
    it.g = ug.x;
    it.n = ug.y;
    it.le = w.tiles[it.g] >> 20;
    return it;
}

// K-blocks of box x (8, or 2 for the last box).
__device__ __forceinline__ int box_blocks(int x) {
    return min(8, kBlocks - 8 * x);
}

__device__ __forceinline__ void arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}

// Stage k of an item is weight box k (8 K-blocks) with the unit's B rows and
// scale blocks of those K-blocks.  Gate/up: issuer 0 multiplies the gate box,
// issuer 1 the up box, each into its accumulator, every stage.  Down: issuer
// k % 2 multiplies stage k into its accumulator and the epilogue adds the two.
// Each issuer copies its stage's scales into a two-slot ring of tensor-memory
// columns; a slot is refilled once the issuer's MMAs that read it completed.
template <bool kGateUp>
__global__ void __launch_bounds__(kThreads, 1) prefill_mma_kernel(LayerDev L, const TmaDesc *tma, PrefillWork w) {
    using S = PSmem<kGateUp>;
    constexpr int kStg = S::kStg;
    constexpr int kBoxA = S::kBoxA;
    extern __shared__ __align__(1024) unsigned char raw[];
    S &s = *reinterpret_cast<S *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int units = *w.unit_count;
    const int items = kScaleTiles * units;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStg; ++i) {
            tc::mbar_init(&s.full[i], 1);
            tc::mbar_init(&s.empty[i], kGateUp ? 2 : 1);
        }
        for (int i = 0; i < 4; ++i) {
            tc::mbar_init(&s.sfree[i >> 1][i & 1], 1);
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
            const uint8_t *bdig = kGateUp ? w.bdig : w.bdig_dn;
            const uint8_t *bsfb = kGateUp ? w.bsfb : w.bsfb_dn;
            for (int i = blockIdx.x; ok && i < items; i += gridDim.x) {
                const Item it = item_of(w, i, units);
                const uint8_t *bu = bdig + size_t(it.u) * kPrefillUnitBytes;
                const uint8_t *su = bsfb + size_t(it.u) * kPrefillUnitScaleBytes;
                for (int k = 0; k < kBoxes; ++k, ++stage) {
                    const uint32_t st = stage % kStg;
                    const uint32_t use = stage / kStg;
                    if (use > 0 && !(ok = wait(&s.empty[st], (use - 1) & 1, w.status))) {
                        break;
                    }
                    const int nchunk = (box_blocks(k) + 3) / 4;
                    // full boxes are counted even where they reach past the matrix (zero fill)
                    const uint32_t tx = uint32_t(kBoxA) * (16384 + uint32_t(nchunk) * kScaleBlockBytes) +
                                        8 * kUnitKbBytes + 4 * kScaleBlockBytes;
                    tc::mbar_expect_tx(&s.full[st], tx);
                    for (int b = 0; b < kBoxA; ++b) {
                        const int map = kGateUp ? (b == 0 ? kTmaGate : kTmaUp) : kTmaDown;
                        const uint8_t *mat = kGateUp ? (b == 0 ? L.gate : L.up) : L.down;
                        tc::tma_load_3d(&s.a[st][b][0], tma + map, 128 * k, 128 * it.mt, it.le, &s.full[st]);
                        bulk(&s.sfa[st][b][0][0], mat + size_t(it.le) * kPackedMatrixBytes + scale_block_offset(it.mt, 2 * k),
                             uint32_t(nchunk) * kScaleBlockBytes, &s.full[st]);
                    }
                    bulk(&s.b[st][0], bu + size_t(8 * k) * kUnitKbBytes, 8 * kUnitKbBytes, &s.full[st]);
                    bulk(&s.sfb[st][0][0][0], su + size_t(2 * k) * 2 * kScaleBlockBytes, 4 * kScaleBlockBytes,
                         &s.full[st]);
                }
            }
            // every load issued has landed before the CTA exits
            for (uint32_t k = 0; k < uint32_t(kStg) && k < stage; ++k) {
                const uint32_t last = stage - 1 - k;
                tc::mbar_wait(&s.full[last % kStg], (last / kStg) & 1);
            }
        }
    } else if (warp >= kIssuerWarp0 && warp < kIssuerWarp0 + 2) {
        if (lane == 0) {
            const int m = warp - kIssuerWarp0;
            const uint32_t dcol = tbase + kColD + uint32_t(kUnitRows) * uint32_t(m);
            uint32_t stage = 0;
            uint32_t mine = 0;  // stages this issuer has multiplied
            uint32_t item_no = 0;
            bool ok = true;
            for (int i = blockIdx.x; ok && i < items; i += gridDim.x, ++item_no) {
                if (item_no > 0 && !(ok = wait(&s.acc_empty, (item_no - 1) & 1, w.status))) {
                    break;
                }
                tc::fence_after_sync();
                const int n = unit_groups(w, i % units).y;
                const uint32_t idesc_n = uint32_t(kGroupRows * n);
                bool first = true;
                for (int k = 0; k < kBoxes; ++k, ++stage) {
                    if (!kGateUp && (k & 1) != m) {
                        continue;  // the other issuer's stage
                    }
                    const uint32_t st = stage % kStg;
                    if (!(ok = wait(&s.full[st], (stage / kStg) & 1, w.status))) {
                        break;
                    }
                    const uint32_t ring = mine & 1;
                    if (mine >= 2 && !(ok = wait(&s.sfree[m][ring], ((mine - 2) >> 1) & 1, w.status))) {
                        break;
                    }
                    tc::fence_after_sync();
                    const int box = kGateUp ? m : 0;
                    const int nkb = box_blocks(k);
                    const int nchunk = (nkb + 3) / 4;
                    const uint32_t sfa_col = tbase + kColSf + 64 * uint32_t(m) + 32 * ring;
                    const uint32_t sfb_col = sfa_col + 8;
                    for (int j = 0; j < nchunk; ++j) {
                        tc::sf_copy(sfa_col + 4 * j, tc::smem_u32(&s.sfa[st][box][j][0]));
                        tc::sf_copy(sfb_col + 8 * j, tc::smem_u32(&s.sfb[st][j][0][0]));
                        if (n > 1) {
                            tc::sf_copy(sfb_col + 8 * j + 4, tc::smem_u32(&s.sfb[st][j][1][0]));
                        }
                    }
                    const uint32_t abase = tc::smem_u32(&s.a[st][box][0]);
                    const uint32_t bbase = tc::smem_u32(&s.b[st][0]);
                    for (int p = 0; 2 * p < nkb; ++p) {
                        const uint32_t sel = uint32_t((2 * p) & 3);
                        const uint32_t j = uint32_t(p >> 1);
                        const uint64_t ad = tc::smem_desc_sw128(abase + 32u * uint32_t(p));
                        const uint64_t bd = tc::smem_desc(bbase + uint32_t(2 * p) * kUnitKbBytes, kUnitKbBytes, 128);
                        tc::mma_f4(dcol, ad, bd, tc::instr_desc_f4(idesc_n, sel), (sfa_col + 4 * j) | (sel << 30),
                                   (sfb_col + 8 * j) | (sel << 30), !first);
                        first = false;
                    }
                    tc::mma_commit(&s.empty[st]);
                    tc::mma_commit(&s.sfree[m][ring]);
                    ++mine;
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
    } else if (warp < 4 || warp >= kEpiWarp1) {
        // epilogue: warps 0-3 take group 0 of the unit, warps 7-10 group 1;
        // thread (quadrant q = warp % 4, lane) is row 32 q + lane of the tile
        // (TMEM lane 32 q + lane)
        const int j = warp < 4 ? 0 : 1;
        const int q = warp & 3;
        uint32_t item_no = 0;
        for (int ii = blockIdx.x; ii < items; ii += gridDim.x, ++item_no) {
            const Item it = item_of(w, ii, units);
            const int row = 128 * it.mt + 32 * q + lane;
            const bool mine = j < it.n;
            float bias0 = 0.0f, bias1 = 0.0f;
            if (mine && row < kDim) {
                if (kGateUp) {
                    bias0 = __ldg(L.gate_b + size_t(it.le) * kDim + row);
                    bias1 = __ldg(L.up_b + size_t(it.le) * kDim + row);
                } else {
                    bias0 = __ldg(L.down_b + size_t(it.le) * kDim + row);
                }
            }
            if (threadIdx.x == 0) {
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
            // each slot's 6 digit columns of both accumulators added up; the
            // accumulators are free once read
            float v0[kGroup], v1[kGroup];
            if (mine) {
                const uint32_t cbase = tbase + (uint32_t(32 * q) << 16) + kColD + uint32_t(kGroupRows * j);
#pragma unroll
                for (int c = 0; c < kGroupRows; c += 48) {
                    float a[48], b[48];
#pragma unroll
                    for (int t = 0; t < 3; ++t) {
                        tc::tmem_ld16(cbase + uint32_t(c + 16 * t), a + 16 * t);
                        tc::tmem_ld16(cbase + uint32_t(kUnitRows + c + 16 * t), b + 16 * t);
                    }
                    tc::wait_ld();
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        float x0 = 0.0f, x1 = 0.0f;
#pragma unroll
                        for (int d = 0; d < kDigits; ++d) {
                            x0 += a[kDigits * t + d];
                            x1 += b[kDigits * t + d];
                        }
                        v0[c / kDigits + t] = x0;
                        v1[c / kDigits + t] = x1;
                    }
                }
            }
            tc::fence_before_sync();
            arrive(&s.acc_empty);
            if (!mine) {
                continue;
            }
            if (kGateUp) {
                // this warp's 32 rows are K-block 4 mt + q of the down product:
                // each slot's 32 values become its 6 digit rows there (zero for
                // padding slots and rows past 2879), and lane s < 16 keeps slot
                // s's block code for the scale bytes
                const int kb = 4 * it.mt + q;
                uint8_t *du = w.bdig_dn + size_t(it.u) * kPrefillUnitBytes + size_t(kb) * kUnitKbBytes +
                              j * kGroupRows * 16;
                uint8_t *su = w.bsfb_dn + size_t(it.u) * kPrefillUnitScaleBytes;
                const int nvalid = group_slots(w, it.g + j).y;
                uint32_t mycode = 0;
#pragma unroll
                for (int slot = 0; slot < kGroup; ++slot) {
                    float h = 0.0f;
                    if (row < kDim && slot < nvalid) {
                        h = swiglu_ref(__fadd_rn(bias0, v0[slot]), __fadd_rn(bias1, v1[slot]));
                    }
                    const uint32_t c = digit_split6_store(h, du + slot * kDigits * 16, lane);
                    mycode = (lane == slot) ? c : mycode;
                }
#pragma unroll
                for (int r = lane; r < kGroupRows; r += 32) {
                    const uint32_t c = __shfl_sync(0xffffffffu, mycode, r / kDigits);
                    su[unit_scale_offset(j * kGroupRows + r, kb)] = uint8_t(digit_scales6(c, r % kDigits));
                }
            } else if (row < kDim) {
                const int2 gs = group_slots(w, it.g + j);
#pragma unroll
                for (int slot = 0; slot < kGroup; ++slot) {
                    if (slot < gs.y) {
                        w.down[size_t(gs.x + slot) * kDim + row] = __fadd_rn(bias0, __fadd_rn(v0[slot], v1[slot]));
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
                         int(sizeof(PSmem<true>) + 1024));
    cudaFuncSetAttribute(prefill_mma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         int(sizeof(PSmem<false>) + 1024));
    cudaFuncSetAttribute(prefill_split_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
}

void launch_prefill_gateup(const LayerDev &L, const TmaDesc *tma, const PrefillWork &w, const PrefillShape &s,
                           const float *x, cudaStream_t stream) {
    const int units = int(prefill_units(size_t(s.tokens), size_t(s.expert_count)));
    prefill_split_kernel<<<std::min(8 * units, 8 * s.sms), 32 * kGroup, 0, stream>>>(w, x);
    prefill_mma_kernel<true><<<s.sms, kThreads, sizeof(PSmem<true>) + 1024, stream>>>(L, tma, w);
}

void launch_prefill_down(const LayerDev &L, const TmaDesc *tma, const PrefillWork &w, const PrefillShape &s,
                         cudaStream_t stream) {
    prefill_mma_kernel<false><<<s.sms, kThreads, sizeof(PSmem<false>) + 1024, stream>>>(L, tma, w);
}

}  // namespace ttl
