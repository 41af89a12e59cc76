// tc.cuh -- 5th-generation tensor core (tcgen05) building blocks for the
// block-scaled MXFP4 x FP8 products of the MoE kernels.
//
// Operands (kind::mxf8f6f4, cta_group::1, M = 128):
//   A = weights, E2M1 with one E8M0 scale per 32 K-elements (the MXFP4 data
//       exactly as stored, no dequantisation): 16 elements per 16-byte
//       shared-memory slot (8 packed bytes, 8 bytes of padding), K-major;
//   B = activations as E4M3 "terms" with their own E8M0 scale per 32 K:
//       x ~= t0 + t1 + t2 + t3, each term captures the residual of the ones
//       before it (4 significant bits each), so 4 terms carry ~16 bits;
//       terms are the N columns of B;
//   D = f32 accumulators in tensor memory (lane = output row, column = term).
// Shared-memory operands use the K-major no-swizzle canonical layout: core
// matrices of 8 rows x 16 bytes (128 contiguous bytes); LBO is the byte
// distance between K-adjacent core matrices, SBO between 8-row groups.
// Scale factors live in tensor memory: per chunk of 4 K-blocks, 4 consecutive
// 32-bit columns; column c + m1, byte k holds the scale of row m0 + 32*m1 for
// K-block k, replicated in all four 32-lane quadrants.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "common.cuh"

namespace ttl {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- tensor memory ----
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(cols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Warp-collective: this warp's 32 lanes, 4 consecutive columns from `taddr`.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}
// Warp-collective: this warp's 32 lanes, 16 consecutive columns from `taddr`.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t a) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(a) : "memory");
}
// Warp-collective: this warp's 32 lanes, 8 consecutive f32 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float v[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = __uint_as_float(r[i]);
    }
}

// ---- mbarrier (bounded waits) ----
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Waits for phase `parity` to complete; gives up after about `limit_ns`
// (default 2 s) and returns false -- the caller records a status bit and
// unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned long long limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) {
        return true;
    }
    const unsigned long long t0 = now_ns();
    while (true) {
        for (int i = 0; i < 64; ++i) {
            if (mbar_try_wait(bar, parity)) {
                return true;
            }
        }
        if (now_ns() - t0 > limit_ns) {
            return false;
        }
    }
}
// Arrives on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// ---- descriptors ----
// K-major, no swizzle.  lbo/sbo in bytes (multiples of 16).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFFu);
    d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
    d |= uint64_t(1) << 46;  // descriptor version for tcgen05
    // base offset 0, lbo mode 0, layout type 0 (no swizzle)
    return d;
}

// K-major, 128-byte swizzle: rows of 128 bytes (eight 16-byte chunks, chunk c
// of row r stored at c ^ (r & 7)), 8-row groups 1024 bytes apart -- the layout
// a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes.  The group must be
// 1024-byte aligned; K-steps inside the 128-byte row advance `saddr`.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFFu);
    d |= uint64_t(1) << 16;            // LBO: unused with a swizzled K-major layout
    d |= uint64_t(1024 >> 4) << 32;    // SBO: 8-row groups
    d |= uint64_t(1) << 46;            // descriptor version for tcgen05
    d |= uint64_t(2) << 61;            // layout type: 128-byte swizzle
    return d;
}

// ---- TMA ----
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Tiled 2-D load of one box of `tmap` at element coordinates (x, y);
// completes the box's bytes on `bar`.  No multicast.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Prefetch of one box of a 2-D `tmap` at (x, y) into L2.  No multicast.
__device__ __forceinline__ void tma_prefetch_2d(const void *tmap, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(x), "r"(y)
                 : "memory");
}

// Tiled 3-D load of one box of `tmap` (a CUtensorMap in global memory) at
// element coordinates (x, y, z); completes `bytes` of the barrier's
// transaction count.  No multicast.
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Prefetch of one box of `tmap` at (x, y, z) into L2 (no shared-memory
// destination, no barrier).  No multicast.
__device__ __forceinline__ void tma_prefetch_3d(const void *tmap, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(tmap), "r"(x), "r"(y),
                 "r"(z)
                 : "memory");
}

// Prefetch of `bytes` contiguous bytes at `src` into L2 (16-byte aligned
// address, size a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 policy for data read once: its lines are the first to be evicted.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// tma_load_3d with an L2 cache policy.
__device__ __forceinline__ void tma_load_3d_hint(void *dst, const void *tmap, int x, int y, int z, uint64_t *bar,
                                                 uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Instruction descriptor: kind::mxf8f6f4, A = E2M1, B = E4M3, scales E8M0,
// K-major A and B, M = 128, N = n.  sfa_id / sfb_id select the scale byte.
__device__ __forceinline__ uint32_t instr_desc(uint32_t n, uint32_t sfa_id, uint32_t sfb_id) {
    uint32_t d = 0;
    d |= (sfb_id & 3u) << 4;
    d |= 5u << 7;             // a_format = E2M1
    d |= 0u << 10;            // b_format = E4M3
    d |= (n >> 3) << 17;      // N >> 3
    d |= 1u << 23;            // scale format E8M0
    d |= (128u >> 4) << 24;   // M >> 4
    d |= (sfa_id & 3u) << 29;
    return d;
}

// D (+)= A x B with block scales; issued by one thread.
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                    uint32_t sfa_tmem, uint32_t sfb_tmem, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
}

// Copies a 32-row x 16-byte scale block from shared memory into 4 tensor-memory
// columns of all four lane quadrants (row m0 -> lane m0 of each quadrant).
// Ordered before later tcgen05.mma of the issuing thread.
__device__ __forceinline__ void sf_copy(uint32_t taddr, uint32_t saddr) {
    const uint64_t d = smem_desc(saddr, 128, 128);
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(d) : "memory");
}

// ---- kind::mxf4 (A and B E2M1, E8M0 scale per 32 K, K = 64 per MMA) ----
// Instruction descriptor: M = 128, N = n, both operands K-major E2M1; sf_id
// (0 or 2) selects the pair of scale bytes (the MMA's two K-blocks).
__device__ __forceinline__ uint32_t instr_desc_f4(uint32_t n, uint32_t sf_id) {
    uint32_t d = 0;
    d |= (sf_id & 3u) << 4;   // B scale byte
    d |= 1u << 7;             // a_format = E2M1
    d |= 1u << 10;            // b_format = E2M1
    d |= (n >> 3) << 17;      // N >> 3
    d |= 1u << 23;            // scale format E8M0
    d |= (128u >> 4) << 24;   // M >> 4
    d |= (sf_id & 3u) << 29;  // A scale byte
    return d;
}
__device__ __forceinline__ void mma_f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa_tmem,
                                       uint32_t sfb_tmem, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// Warp-collective: this warp's 32 lanes, 16 consecutive f32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v[i] = __uint_as_float(r[i]);
    }
}

// ---- activation digits (the B operand of the kind::mxf4 products) ----
// The 32 values of one K-block (one per lane) in block fixed point: with e the
// exponent of the block's largest magnitude, |v| = m * 2^(e-23), m < 2^24
// rounded to nearest, written as 12 base-4 digits m = sum_n d_n 4^n.  Digit n
// is the E2M1 value 0, 1, 2 or 3 with the sign of v -- row n of B -- and its
// E8M0 scale is 2^(e - 23 + 2n).  Values below 2^(e-24) of the block's
// largest are rounded away; nothing else is lost.
constexpr int kDigitTerms = 12;

// E2M1 codes of eight 2-bit digits held in the low bits of each nibble of x
// (0 -> 0, 1 -> 1.0, 2 -> 2.0, 3 -> 3.0), with the sign bit on nonzero digits.
__device__ __forceinline__ uint32_t digit_codes(uint32_t x, uint32_t negative) {
    const uint32_t b0 = x & 0x11111111u;
    const uint32_t b1 = (x >> 1) & 0x11111111u;
    const uint32_t code = (b1 << 2) | (b0 & b1) | ((b0 & ~b1) << 1);
    return code | (((b0 | b1) << 3) & (0u - negative));
}

// Eight 2-bit fields of the low 16 bits of v, one per nibble.
__device__ __forceinline__ uint32_t spread_digits(uint32_t v) {
    v &= 0xFFFFu;
    v = (v | (v << 8)) & 0x00FF00FFu;
    v = (v | (v << 4)) & 0x0F0F0F0Fu;
    return (v | (v << 2)) & 0x33333333u;
}

// Lane l holds 8 nibbles (element l, rows 0..7); afterwards lane l holds row
// (l & 7) of elements 8*(l >> 3) .. +7 (nibble j = element 8*(l >> 3) + j).
__device__ __forceinline__ uint32_t transpose_nibbles(uint32_t x, int lane) {
    uint32_t t = __shfl_xor_sync(0xffffffffu, x, 4);
    x = (lane & 4) ? ((x & 0xFFFF0000u) | (t >> 16)) : ((x & 0x0000FFFFu) | (t << 16));
    t = __shfl_xor_sync(0xffffffffu, x, 2);
    x = (lane & 2) ? ((x & 0xFF00FF00u) | ((t >> 8) & 0x00FF00FFu)) : ((x & 0x00FF00FFu) | ((t << 8) & 0xFF00FF00u));
    t = __shfl_xor_sync(0xffffffffu, x, 1);
    x = (lane & 1) ? ((x & 0xF0F0F0F0u) | ((t >> 4) & 0x0F0F0F0Fu)) : ((x & 0x0F0F0F0Fu) | ((t << 4) & 0xF0F0F0F0u));
    return x;
}

// Splits one K-block (warp-collective, one value per lane) and writes its B
// rows into `kb_base` ([2 row groups][8 rows][16 B]; rows 12..15 are written
// as zero).  Returns the block code e + 127 (127 for an all-zero block, 255
// for a block holding inf or NaN: its row scales become the E8M0 NaN and the
// products carry the NaN on).  kb_base may be shared or global memory.
__device__ __forceinline__ uint32_t digit_split_store(float v, uint8_t *kb_base, int lane) {
    const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
    uint32_t code, m = 0u;
    if (mb >= 0x7f800000u) {
        code = 255u;
    } else if (mb == 0u || int(mb >> 23) < 27) {  // zero, or every |v| below 2^-100
        code = 127u;
    } else {
        const int e = int(mb >> 23) - 127;
        m = __float2uint_rn(__fmul_rn(fabsf(v), __uint_as_float(uint32_t(150 - e) << 23)));  // |v| * 2^(23-e)
        code = uint32_t(e + 127);
    }
    const uint32_t neg = __float_as_uint(v) >> 31;
    const uint32_t lo = transpose_nibbles(digit_codes(spread_digits(m), neg), lane);
    const uint32_t hi = transpose_nibbles(digit_codes(spread_digits(m >> 16), neg), lane);
    const int off = (lane & 7) * 16 + 4 * (lane >> 3);
    *reinterpret_cast<uint32_t *>(kb_base + off) = lo;
    *reinterpret_cast<uint32_t *>(kb_base + 128 + off) = hi;
    return code;
}

// Scale bytes of B row `row` for four K-blocks' codes (one per byte).
__device__ __forceinline__ uint32_t digit_scales4(uint32_t codes4, int row) {
    if (row >= kDigitTerms) {
        return 0x7F7F7F7Fu;
    }
    const uint32_t v = __vsubus4(codes4, uint32_t(23 - 2 * row) * 0x01010101u);
    const uint32_t nan = __vcmpeq4(codes4, 0xFFFFFFFFu);
    return (v & ~nan) | nan;
}

// ---- activation terms ----
// Splits the 32 values of one K-block (one per lane) into kTerms E4M3 terms
// with one E8M0 scale each: returns this lane's term bytes packed in a u32
// (term j in byte j) and writes the scale bytes to scales (lane 0's view).
template <int kTerms>
__device__ __forceinline__ uint32_t split_terms(float v, uint32_t &scale_bytes) {
    uint32_t bytes = 0;
    scale_bytes = 0;
    float r = v;
#pragma unroll
    for (int j = 0; j < kTerms; ++j) {
        // block max of |r| (non-negative floats order like their bit patterns)
        const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(r)));
        const float m = __uint_as_float(mb);
        // scale 2^(E-7) where 2^E <= m < 2^(E+1): m / scale in [128, 256) <= 448
        int e8 = 127;
        if (m > 0.0f && m == m) {
            const int E = int((mb >> 23) & 0xFF) - 127;
            e8 = E - 7 + 127;
            e8 = e8 < 1 ? 1 : (e8 > 253 ? 253 : e8);
        }
        const float inv = __uint_as_float(uint32_t(254 - e8) << 23);  // 2^-(e8-127), exact
        const float sc = __uint_as_float(uint32_t(e8) << 23);
        const __nv_fp8_e4m3 q(__fmul_rn(r, inv));
        const float back = __fmul_rn(float(q), sc);
        r = __fsub_rn(r, back);
        bytes |= uint32_t(q.__x) << (8 * j);
        scale_bytes |= uint32_t(e8) << (8 * j);
    }
    return bytes;
}

} // namespace tc
} // namespace ttl
