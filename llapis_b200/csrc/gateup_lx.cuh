// gate_up grouped GEMM of the prefill path, bit-exact with the reference's CPU dots.
//
// ggml-cpu's x86 kernels for the gate_up types (ggml_vec_dot_q4_K_q8_K, x86/quants.c:1900;
// _iq2_s_q8_K :2937; _iq2_xxs_q8_K :2522) fix the float order of every dot: per 256-value
// super-block, eight integer lanes (lane L sums the products at positions 4L..4L+3 of each 32-value
// group, the sub-block scale inside the integer), each lane fused-multiply-added into its own f32
// accumulator with the super-block's scale d = d_x * d_w, and at the end the horizontal sum
// ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)) (hsum_float_8, :43). Q4_K adds a min term of
// four lanes (mins[2m] * q8s[2m] + mins[2m+1] * q8s[2m+1], q8s the 32-value sub-block sums), fused
// into its own four accumulators with dmin = -d_x * dmin_w, reduced as (m0 + m2) + (m1 + m3) and
// added last. A last-bit difference here moves the Q8_0 and fp16-GELU roundings of the down input,
// so this kernel reproduces that order exactly:
//
//   - the tensor cores compute each lane's exact integer sum (kind::f16 with small-integer fp16
//     operands, fp32 accumulation of integers below 2^24), one accumulator per lane;
//   - a "pass" runs two lanes over all super-blocks of the row: (0,4), (2,6), (1,5), (3,7), then for
//     Q4_K the min lanes (0,2), (1,3); the epilogue keeps the two lanes' f32 chains in registers
//     (fma.rn.f32x2 per column pair) and folds finished passes into two held partial sums in the
//     reference's reduction order;
//   - operands: A = the weight rows (M = 128: 64 gate + 64 up rows), converted by four warps (thread
//     = row = TMEM lane) and stored straight into tensor memory with tcgen05.st (no shared-memory
//     round trip); B = the pairs' Q8_K values as fp16, in a per-(tile, pass, super-block) image that
//     pf_gather_lx_kernel lays out in the same lane order, bulk-copied into shared memory by a
//     producer warp up to four steps ahead; N = up to 64 pairs per work unit.
//
// TMEM (512 columns): three accumulator buffers of 2 lanes x 64 columns [0, 384) and four A buffers
// of 32 columns [384, 512); the two held partial sums live in shared memory.
#pragma once

namespace moeb {

constexpr int kLxN = 64;                    // pairs per work unit (MMA N <= 64)
constexpr int kLxMainCores = 8;             // K = 64 per main pass step (2 lanes x 32), in 8-value cores
constexpr int kLxBStageBytes = (kLxN / 8) * kLxMainCores * 128;   // 8 KB: one unit's half of a main image
constexpr int kLxEpiWarps = 16;             // four per TMEM lane quadrant, 16 columns each
constexpr int kLxEpiCols = kLxN / (kLxEpiWarps / 4);
constexpr int kLxConvGroups = 2;            // converter groups of four warps (one per TMEM lane quadrant),
constexpr int kLxConvWarps = 4 * kLxConvGroups;   // group g converting steps g, g + groups, ...
constexpr int kLxEpiWarp0 = kLxConvWarps;
// MMA issue and operand copies: kLxIssue warps each, taking alternate steps, so that their issue
// work is spread over the four SM sub-partitions instead of slowing the epilogue warps of two
constexpr int kLxIssue = 2;
constexpr int kLxMmaWarp = kLxEpiWarp0 + kLxEpiWarps;
constexpr int kLxProdWarp = kLxMmaWarp + kLxIssue;
constexpr int kLxThreads = (kLxProdWarp + kLxIssue) * 32;
// TMEM: three accumulator buffers of 2 lanes x 64 columns, then four A buffers of 32 columns; the
// A buffers and the B stages share one ring index (step % kLxRing) and one "operands free" barrier
constexpr int kLxDBufs = 3, kLxRing = 4;
constexpr uint32_t kLxColD = 0, kLxColA = 128 * kLxDBufs, kLxTmemCols = 512;
static_assert(kLxColA + 32 * kLxRing <= kLxTmemCols, "TMEM budget");
static_assert(kLxImgMain == (kPrefillTile / 8) * kLxMainCores * 128, "image size in params.h");

// the two reference lanes of main pass p: (0,4), (2,6), (1,5), (3,7)
MOEB_HD constexpr int lx_first_lane(int pass) { return pass == 0 ? 0 : pass == 1 ? 2 : pass == 2 ? 1 : 3; }
template <int PASS>
__device__ constexpr int lx_lane_c(int second) { return lx_first_lane(PASS) + 4 * second; }

// Q4_K raw row blocks of a step, staged by two 2D tensor-map copies (64 gate rows, 64 up rows) of
// 144 bytes (one super-block) per row
constexpr int kLxRawBytes = kPfM * B_Q4_K;
struct LxMaps {
    CUtensorMap gu[2];   // [hot, cold] gate_up pools as 2D byte arrays (row bytes x rows); Q4_K pools only
};
struct LxSmem {
    uint8_t b[kLxRing][kLxBStageBytes];
    uint8_t raw[kLxRing][kLxRawBytes];       // Q4_K units: the step's super-block of the unit's 128 rows
    float held[2][kLxN][kPfM];               // the two held partial sums of each (row, column), column-major
    float dxs[kPrefillMaxSb][kLxN];          // Q8_K scale of each unit column, per super-block
    float xdt[kPrefillMaxSb][kPfM];          // d_w of each unit row, per super-block
    uint64_t bfull[kLxRing], afull[kLxRing], opfree[kLxRing], dfull[kLxDBufs], dempty[kLxDBufs], done, epibar;
    uint32_t tmem;
    int32_t abort;
};

// ---------------------------------------------------------------- TMEM stores / loads of 32-bit columns
#define MOEB_R32(a) MOEB_R16(a), "=r"(a[16]), "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), \
    "=r"(a[22]), "=r"(a[23]), "=r"(a[24]), "=r"(a[25]), "=r"(a[26]), "=r"(a[27]), "=r"(a[28]), "=r"(a[29]), "=r"(a[30]), \
    "=r"(a[31])
#define MOEB_I16(a) "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(a[8]), \
    "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]), "r"(a[15])
#define MOEB_I32(a) MOEB_I16(a), "r"(a[16]), "r"(a[17]), "r"(a[18]), "r"(a[19]), "r"(a[20]), "r"(a[21]), "r"(a[22]), \
    "r"(a[23]), "r"(a[24]), "r"(a[25]), "r"(a[26]), "r"(a[27]), "r"(a[28]), "r"(a[29]), "r"(a[30]), "r"(a[31])

__device__ __forceinline__ void tmem_st16(uint32_t ta, const uint32_t (&v)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 ::"r"(ta), MOEB_I16(v) : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t ta, const uint32_t (&v)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
                 ::"r"(ta), MOEB_I32(v) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t ta, uint32_t (&v)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                 "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : MOEB_R32(v) : "r"(ta));
    asm volatile("tcgen05.wait::ld.sync.aligned;" : MOEB_RW16(v), "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]),
                 "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]), "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]),
                 "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])::"memory");
}
// 16 columns of two accumulators (lane a and lane b of a pass) in one wait
__device__ __forceinline__ void tmem_ld16x2u(uint32_t ta, uint32_t tb, uint32_t (&a)[16], uint32_t (&b)[16]) {
    asm volatile(MOEB_LD16 : MOEB_R16(a) : "r"(ta));
    asm volatile(MOEB_LD16 : MOEB_R16(b) : "r"(tb));
    asm volatile("tcgen05.wait::ld.sync.aligned;" : MOEB_RW16(a), MOEB_RW16(b)::"memory");
}

// 8 columns of two accumulators in one wait
#define MOEB_LD8 "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
__device__ __forceinline__ void tmem_ld8x2u(uint32_t ta, uint32_t tb, uint32_t (&a)[8], uint32_t (&b)[8]) {
    asm volatile(MOEB_LD8 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7])
                 : "r"(ta));
    asm volatile(MOEB_LD8 : "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7])
                 : "r"(tb));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), "+r"(b[0]),
                   "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])::"memory");
}

// MMA with the A operand in tensor memory (M = 128 rows in the 128 TMEM lanes, K along the
// columns, two fp16 values per 32-bit column) and B from shared memory
__device__ __forceinline__ void umma_f16_ts(uint32_t dtmem, uint32_t atmem, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(dtmem),
        "r"(atmem), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}

// ---------------------------------------------------------------- packed f32 pairs (IEEE, round to nearest)
__device__ __forceinline__ uint64_t f2pack(float x, float y) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
    return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// ---------------------------------------------------------------- waits that sleep
// mbarrier.try_wait with a suspend-time hint: a waiting thread is suspended until the phase completes
// (or the hint of ~1 us runs out) instead of spinning, so waiting warps leave the issue slots to the
// converters, the MMA thread and the epilogue. Bounded like pf_wait: after kLxWaitLimit tries (about
// a second) the wait records ERR_MBAR_TIMEOUT, raises the CTA's abort flag and gives up.
constexpr uint32_t kLxWaitLimit = 1u << 20;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool lx_wait(uint64_t *bar, uint32_t parity, volatile int32_t *abort) {
    for (uint32_t i = 0; i < kLxWaitLimit; ++i) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if ((i & 15u) == 15u && *abort) return false;
    }
    atomicOr(&g_error, ERR_MBAR_TIMEOUT);
    *abort = 1;
    return false;
}
__device__ __forceinline__ bool lx_wait_warp(uint64_t *bar, uint32_t parity, volatile int32_t *abort) {
    return __all_sync(0xffffffffu, lx_wait(bar, parity, abort));
}
// One lane of a converged warp (elect.sync): the single-thread issue points (MMA, commit, bulk copy)
// sit inside warp-uniform loops, so their operands stay in uniform registers.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------- 2D tensor-map copy (no multicast)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// ---------------------------------------------------------------- A operands (weight rows, one thread per row)
// Lane L's 32 values of a super-block in K order 4j + e <-> value 32j + 4L + e (j = 32-value
// group, e < 4): 16 columns of fp16 pairs.

// Q4_K (block: d, dmin, scales[12], qs[128]; byte 32c + b holds value b of sub-block 2c in its low
// nibble and of sub-block 2c + 1 in its high nibble): A = sc_j * q, exact in fp16
__device__ __forceinline__ void lx_a_q4k_lane(const uint32_t (&qw)[4], const __half2 (&s2)[8], const __half2 (&ns2)[8],
                                              uint32_t *o) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        scale4(qw[c] & 0x0f0f0f0fu, s2[2 * c], ns2[2 * c], o[4 * c], o[4 * c + 1]);
        scale4((qw[c] >> 4) & 0x0f0f0f0fu, s2[2 * c + 1], ns2[2 * c + 1], o[4 * c + 2], o[4 * c + 3]);
    }
}

// The eight 6-bit scales (mins) of a Q4_K super-block as bytes of two words (get_scale_min_k4,
// ggml-quants.c:822), from the scale words w1, w2, w3 (bytes 4..15 of the block)
__device__ __forceinline__ void q4k_scale_words(uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&sc)[2], uint32_t (&mn)[2]) {
    sc[0] = w1 & 0x3f3f3f3fu;
    sc[1] = (w3 & 0x0f0f0f0fu) | ((w1 >> 2) & 0x30303030u);
    mn[0] = w2 & 0x3f3f3f3fu;
    mn[1] = ((w3 >> 4) & 0x0f0f0f0fu) | ((w2 >> 2) & 0x30303030u);
}
// byte j of two words as an exact fp16 pair (v, v): bytes [v, 0x64, v, 0x64] are (1024 + v) twice
__device__ __forceinline__ __half2 byte_h2(const uint32_t (&w)[2], int j) {
    const uint32_t b = (uint32_t)(j & 3);
    return __hsub2(u2h(__byte_perm(w[j >> 2], 0x64646464u, 0x4040u | b | (b << 8))), u2h(0x64006400u));
}

// IQ2_S (block: d, qs[32] grid low bytes, signs[32], qh[8], scales[8]): value 32b + 4L + e is byte
// 4(L & 1) + e of grid entry g = 4b + L/2 (index qs[g] | 2 bits of qh[b]), sign bit of signs[g],
// times ls = 2 * (L < 4 ? low : high scale nibble of block b) + 1
__device__ __forceinline__ void lx_a_iq2s_lane(const uint8_t *blk, int L, uint32_t *o) {
    const uint8_t *qs = blk + 2, *sg = blk + 34, *qh = blk + 66, *scl = blk + 74;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const int g = 4 * b + (L >> 1);
        const uint32_t idx = (uint32_t)__ldg(qs + g) | ((((uint32_t)__ldg(qh + b) >> (2 * (g & 3))) & 3u) << 8);
        const uint64_t grid = g_iq2s_grid[idx];
        const uint32_t mag = (uint32_t)(grid >> (32 * (L & 1)));
        const uint32_t sv = __ldg(scl + b);
        const int ls = 2 * (int)(L < 4 ? (sv & 0xfu) : (sv >> 4)) + 1;
        const __half2 s2 = __float2half2_rn((float)ls), ns2 = __float2half2_rn(-1024.f * ls);
        uint32_t o0, o1;
        scale4(mag, s2, ns2, o0, o1);
        const uint32_t s4 = ((uint32_t)__ldg(sg + g) >> (4 * (L & 1))) & 0xfu;
        o0 ^= ((s4 & 1u) << 15) | ((s4 & 2u) << 30);
        o1 ^= ((s4 & 4u) << 13) | ((s4 & 8u) << 28);
        o[2 * b] = o0;
        o[2 * b + 1] = o1;
    }
}

// IQ2_XXS (block: d, then per 32-block 4 grid indices and a u32 of four 7-bit sign indices + a 4-bit
// scale): value 32b + 4L + e is byte 4(L & 1) + e of grid entry aux[L/2], the sign from the 7-bit
// index's pattern, times 2 * ls + 1
__device__ __forceinline__ void lx_a_iq2xxs_lane(const uint8_t *blk, int L, uint32_t *o) {
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const uint8_t *g8 = blk + 2 + 8 * b;
        const uint32_t hi = (uint32_t)__ldg(g8 + 4) | ((uint32_t)__ldg(g8 + 5) << 8) | ((uint32_t)__ldg(g8 + 6) << 16) |
                            ((uint32_t)__ldg(g8 + 7) << 24);
        const int l = L >> 1;
        const uint64_t grid = g_iq2xxs_grid[__ldg(g8 + l)];
        const uint32_t mag = (uint32_t)(grid >> (32 * (L & 1)));
        const int ls = 2 * (int)(hi >> 28) + 1;
        const __half2 s2 = __float2half2_rn((float)ls), ns2 = __float2half2_rn(-1024.f * ls);
        uint32_t o0, o1;
        scale4(mag, s2, ns2, o0, o1);
        const uint32_t s4 = ((uint32_t)g_iq2xxs_signs[(hi >> (7 * l)) & 127u] >> (4 * (L & 1))) & 0xfu;
        o0 ^= ((s4 & 1u) << 15) | ((s4 & 2u) << 30);
        o1 ^= ((s4 & 4u) << 13) | ((s4 & 8u) << 28);
        o[2 * b] = o0;
        o[2 * b + 1] = o1;
    }
}

// ---------------------------------------------------------------- B operand images
// One CTA per (tile, super-block), thread = (tile row c, half h): half 0 writes main passes 0, 1
// (lanes (0,4), (2,6)), half 1 passes 2, 3 ((1,5), (3,7)). An image row holds lane a's 32 values
// (cores 0-3) then lane b's (cores 4-7), each in K order 4j + e. Rows n..N-1 (padding up to a
// multiple of 16) are zero. Half 0 also writes the row's Q8_K scale, half 1 its 16 bsums as fp16
// pairs (exact: |bsum| <= 16 x 127) for pf_q4k_min_kernel.
template <int PASS>
__device__ __forceinline__ void lx_b_main_row(const uint4 (&v)[16], uint8_t *img, int c) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int L = j < 4 ? lx_lane_c<PASS>(0) : lx_lane_c<PASS>(1);
        const int g0 = 2 * (j & 3);   // 32-value groups g0, g0 + 1 in this core
        uint32_t w[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int wi = 8 * (g0 + q) + L;   // word index of values 32(g0+q) + 4L .. + 3
            const uint4 &u = v[wi >> 2];
            w[q] = (wi & 3) == 0 ? u.x : (wi & 3) == 1 ? u.y : (wi & 3) == 2 ? u.z : u.w;
        }
        uint32_t o0, o1, o2, o3;
        s8x4_h(w[0], o0, o1);
        s8x4_h(w[1], o2, o3);
        *reinterpret_cast<uint4 *>(img + canon_off(c, j, kLxMainCores)) = make_uint4(o0, o1, o2, o3);
    }
}

__global__ void __launch_bounds__(256) pf_gather_lx_kernel(PfParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const int ti = blockIdx.x, sb = blockIdx.y;
    if (ti >= *p.n_tiles) return;
    const PfTile tl = p.tiles[ti];
    const int N = (tl.n + 15) & ~15, nsb = p.d / QK_K;
    const int c = threadIdx.x >> 1, h = threadIdx.x & 1;
    if (c >= N) return;
    uint8_t *base = p.bimg + (size_t)ti * lx_tile_bytes(nsb);
    uint8_t *im0 = base + lx_image_off(nsb, 2 * h, sb), *im1 = base + lx_image_off(nsb, 2 * h + 1, sb);
    float *dxt = p.dxt + ((size_t)ti * nsb + sb) * kPfN;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    if (c >= tl.n) {
#pragma unroll
        for (int j = 0; j < kLxMainCores; ++j) {
            *reinterpret_cast<uint4 *>(im0 + canon_off(c, j, kLxMainCores)) = z;
            *reinterpret_cast<uint4 *>(im1 + canon_off(c, j, kLxMainCores)) = z;
        }
        if (h == 0) dxt[c] = 0.f;
        return;
    }
    uint4 *bst = reinterpret_cast<uint4 *>(p.bst + (((size_t)ti * nsb + sb) * kPfN + c) * 8);
    const int t = p.perm[tl.slot0 + c] / p.k;
    const int8_t *q8 = p.xq8 + (size_t)t * p.d + sb * QK_K;
    uint4 v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __ldg(reinterpret_cast<const uint4 *>(q8 + 16 * i));
    if (h == 0) {
        lx_b_main_row<0>(v, im0, c);
        lx_b_main_row<1>(v, im1, c);
        dxt[c] = p.xd[(size_t)t * nsb + sb];
    } else {
        lx_b_main_row<2>(v, im0, c);
        lx_b_main_row<3>(v, im1, c);
        const uint4 *bs = reinterpret_cast<const uint4 *>(p.xbs + ((size_t)t * nsb + sb) * 16);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint4 u = __ldg(bs + i);
            const uint32_t raw[4] = {u.x, u.y, u.z, u.w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = pack_h2i((int)(int16_t)(raw[j] & 0xffffu), (int)(int16_t)(raw[j] >> 16));
            bst[i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// ---------------------------------------------------------------- Q4_K min term, M = (m0 + m2) + (m1 + m3)
// The four min lanes of ggml_vec_dot_q4_K_q8_K (x86/quants.c:1900): per super-block, lane m is the
// integer mins[2m] * q8s[2m] + mins[2m+1] * q8s[2m+1] (q8s[j] = bsums[2j] + bsums[2j+1]), fused into
// its own f32 chain with dmin = -d_x * dmin_w; the four chains reduce as (m0 + m2) + (m1 + m3), which
// the dot adds last. This kernel computes M for every (row, pair) of the Q4_K tiles and stores it in
// hbuf, where the grouped GEMM's epilogue adds the main lanes' sum to it.
//
// The integers come from mma.sync m16n8k8 (fp16 operands, f32 accumulators, all exact) with the
// lanes in M: for a weight row, M-row g holds lane 0 (2) and M-row g + 8 lane 1 (3) of the low (high)
// half of the 16 bsums; lane m's two mins sit twice each at the K of its four bsums and zeros
// elsewhere, B column c is the pair's eight bsums of that half, so two MMAs give all four lane
// integers of 8 rows x 8 pairs and every (row, pair) chain stays in one thread's registers. CTA = (tile, 128 rows), eight warps of 16 rows; the tile's bsums (fp16 pairs, written
// by pf_gather_lx_kernel) and scales are staged once, then 32-pair chunks (four n-blocks) run.
// (A packed-f32 CUDA-core formulation of the same integers measured slower here: its operand tables
// make it shared-memory bound.)
constexpr int kMinRows = 128, kMinCols = 32, kMinThreads = 256;
// dynamic shared memory: per super-block the tile's bsums [128][8] + scales [128] and the CTA rows'
// mins [128] (uint2) + -dmin_w [128]
MOEB_HD constexpr size_t min_smem_bytes(int nsb) { return (size_t)nsb * (kPfN * 36 + kMinRows * 12); }
__device__ __forceinline__ void mma_f16_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
                 : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0), "f"(0.f));
}

__global__ void __launch_bounds__(kMinThreads) pf_q4k_min_kernel(PfParams p) {
    extern __shared__ __align__(16) uint8_t mn_smem[];
    pdl_wait();
    pdl_launch_dependents();
    const int ti = blockIdx.x, rb = blockIdx.y;
    if (ti >= *p.n_tiles) return;
    const PfTile tl = p.tiles[ti];
    const bool c1 = tl.cls != 0;
    PoolView pv;
    pv.w = c1 ? p.gu[1].w : p.gu[0].w;
    pv.type = c1 ? p.gu[1].type : p.gu[0].type;
    pv.ptrs = c1 ? p.gu[1].ptrs : p.gu[0].ptrs;
    if (pv.type != T_Q4_K) return;
    const int nsb = p.d / QK_K, gu_rows = 2 * p.nff, row0 = rb * kMinRows;
    const int N = (tl.n + kMinCols - 1) / kMinCols * kMinCols;
    uint32_t(*s_bs)[kPfN][8] = reinterpret_cast<uint32_t(*)[kPfN][8]>(mn_smem);
    float(*s_dx)[kPfN] = reinterpret_cast<float(*)[kPfN]>(mn_smem + (size_t)nsb * kPfN * 32);
    uint2(*s_mins)[kMinRows] = reinterpret_cast<uint2(*)[kMinRows]>(mn_smem + (size_t)nsb * kPfN * 36);
    float(*s_ndmin)[kMinRows] = reinterpret_cast<float(*)[kMinRows]>(mn_smem + (size_t)nsb * (kPfN * 36 + kMinRows * 8));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    // the tile's bsums and scales, columns [0, N) (those at or past the tile's n are never stored)
    for (int i = tid; i < nsb * N * 2; i += kMinThreads) {
        const int sb = i / (N * 2), rem = i - sb * N * 2;
        reinterpret_cast<uint4 *>(&s_bs[sb][0][0])[rem] =
            reinterpret_cast<const uint4 *>(p.bst + ((size_t)ti * nsb + sb) * kPfN * 8)[rem];
    }
    for (int i = tid; i < nsb * N; i += kMinThreads) {
        const int sb = i / N, c = i - sb * N;
        s_dx[sb][c] = p.dxt[((size_t)ti * nsb + sb) * kPfN + c];
    }
    // the CTA rows' block headers: mins and -dmin_w
    const uint8_t *base = tile_rows(pv, tl.widx, gu_rows, p.d);
    const size_t rbytes = row_bytes(T_Q4_K, p.d);
    for (int i = tid; i < nsb * kMinRows; i += kMinThreads) {
        const int sb = i / kMinRows, r = i - sb * kMinRows;
        const uint4 h = __ldg(reinterpret_cast<const uint4 *>(base + (size_t)(row0 + r) * rbytes + (size_t)sb * B_Q4_K));
        uint32_t sc[2], mn[2];
        q4k_scale_words(h.y, h.z, h.w, sc, mn);
        s_mins[sb][r] = make_uint2(mn[0], mn[1]);
        s_ndmin[sb][r] = -h2f((uint16_t)(h.x >> 16));
    }
    __syncthreads();
    const int ra = 16 * warp + g, rbw = ra + 8;   // this thread's two rows (of the CTA's 128)
    const bool lo = t4 < 2;
    for (int c0 = 0; c0 < N; c0 += kMinCols) {
        float acc[4][4][4];   // [n-block][lane m][fragment element]
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int m = 0; m < 4; ++m)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[j][m][e] = 0.f;
        for (int sb = 0; sb < nsb; ++sb) {
            const uint2 ma = s_mins[sb][ra], mb = s_mins[sb][rbw];
            const uint32_t wa[2] = {ma.x, ma.y}, wb[2] = {mb.x, mb.y};
            // m16n8k8 with the lanes in M: for weight row r, M-row g holds lane 2h (low MMA, bsums 0..7)
            // or lane 2h + 2 (high MMA, bsums 8..15) and M-row g + 8 the next lane; lane m's two mins
            // sit at the K of its four bsums (each min twice), zeros elsewhere, so B needs no mask
            const uint32_t vla = h2u(byte_h2(wa, t4)), vha = h2u(byte_h2(wa, t4 + 4));
            const uint32_t vlb = h2u(byte_h2(wb, t4)), vhb = h2u(byte_h2(wb, t4 + 4));
            const uint32_t la0 = lo ? vla : 0u, la1 = lo ? 0u : vla, ha0 = lo ? vha : 0u, ha1 = lo ? 0u : vha;
            const uint32_t lb0 = lo ? vlb : 0u, lb1 = lo ? 0u : vlb, hb0 = lo ? vhb : 0u, hb1 = lo ? 0u : vhb;
            const float nda = s_ndmin[sb][ra], ndb = s_ndmin[sb][rbw];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int cb = c0 + 8 * j;
                // B: column g of n-block j, K 2t4, 2t4+1 = bsums 2t4, 2t4+1 (low) or 8 + 2t4, 9 + 2t4 (high)
                const uint32_t p0 = s_bs[sb][cb + g][t4], p1 = s_bs[sb][cb + g][t4 + 4];
                const float2 dx = *reinterpret_cast<const float2 *>(&s_dx[sb][cb + 2 * t4]);
                // dmin = -d_x * dmin_w per (row, pair), rounded to f32
                const float dm[4] = {__fmul_rn(dx.x, nda), __fmul_rn(dx.y, nda), __fmul_rn(dx.x, ndb), __fmul_rn(dx.y, ndb)};
                float dl[4], dh[4];
                // row ra: lanes 0, 1 (low) and 2, 3 (high); fragment rows g / g + 8 = the two lanes
                mma_f16_1688(dl, la0, la1, p0);
                mma_f16_1688(dh, ha0, ha1, p1);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    acc[j][0][q] = __fmaf_rn(dm[q], dl[q], acc[j][0][q]);
                    acc[j][1][q] = __fmaf_rn(dm[q], dl[2 + q], acc[j][1][q]);
                    acc[j][2][q] = __fmaf_rn(dm[q], dh[q], acc[j][2][q]);
                    acc[j][3][q] = __fmaf_rn(dm[q], dh[2 + q], acc[j][3][q]);
                }
                // row rbw
                mma_f16_1688(dl, lb0, lb1, p0);
                mma_f16_1688(dh, hb0, hb1, p1);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    acc[j][0][2 + q] = __fmaf_rn(dm[2 + q], dl[q], acc[j][0][2 + q]);
                    acc[j][1][2 + q] = __fmaf_rn(dm[2 + q], dl[2 + q], acc[j][1][2 + q]);
                    acc[j][2][2 + q] = __fmaf_rn(dm[2 + q], dh[q], acc[j][2][2 + q]);
                    acc[j][3][2 + q] = __fmaf_rn(dm[2 + q], dh[2 + q], acc[j][3][2 + q]);
                }
            }
        }
        // fragment element e: row (e < 2 ? g : g + 8), pair 2 t4 + (e & 1) of the n-block
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = c0 + 8 * j + 2 * t4 + (e & 1);
                if (c >= tl.n) continue;
                const float M = __fadd_rn(__fadd_rn(acc[j][0][e], acc[j][2][e]), __fadd_rn(acc[j][1][e], acc[j][3][e]));
                const int wr = row0 + (e < 2 ? ra : rbw);
                p.hbuf[(size_t)(tl.slot0 + c) * gu_rows + wr] = M;
            }
    }
}

// ---------------------------------------------------------------- the grouped GEMM
// Work unit (tile, mb, nh): 64 gate rows [64 mb, 64 mb + 64) and the matching 64 up rows against
// pairs [64 nh, 64 nh + 64) of an expert tile (units of an empty half are skipped by every role
// alike). Persistent: CTA b takes units b, b + grid, ...; a step is (unit, pass, super-block), and
// every role walks the same step sequence with an LxIter.
__device__ __forceinline__ bool lx_unit(const PfParams &p, int u, int n_mb, int &ti, int &mb, int &nh, PfTile &tl) {
    ti = u / (2 * n_mb);
    const int rem = u - ti * 2 * n_mb;
    mb = rem >> 1;
    nh = rem & 1;
    tl = p.tiles[ti];
    return 64 * nh < tl.n;
}
__device__ __forceinline__ int lx_passes(int) { return 4; }

struct LxIter {
    int u, ti, mb, nh, pass, sb, np, nc, N, type;
    PfTile tl;
    const uint8_t *arow;   // this thread's weight row of the unit (rows 0..63 gate, 64..127 the matching up rows)
    bool ok;
    // from u (inclusive): the first unit with pairs in it; r: this thread's row (< 0: no row)
    __device__ __forceinline__ void seek(const PfParams &p, int units, int n_mb, int r) {
        for (; u < units; u += gridDim.x)
            if (lx_unit(p, u, n_mb, ti, mb, nh, tl)) break;
        ok = u < units;
        if (ok) {
            // field by field, not p.gu[tl.cls]: a runtime index into the parameter block copies it to
            // local memory
            const bool c1 = tl.cls != 0;
            PoolView pv;
            pv.w = c1 ? p.gu[1].w : p.gu[0].w;
            pv.type = c1 ? p.gu[1].type : p.gu[0].type;
            pv.ptrs = c1 ? p.gu[1].ptrs : p.gu[0].ptrs;
            type = pv.type;
            np = lx_passes(type);
            nc = min(kLxN, tl.n - 64 * nh);
            N = (nc + 15) & ~15;
            pass = 0;
            sb = 0;
            if (r >= 0) {
                const int wr = r < 64 ? 64 * mb + r : p.nff + 64 * mb + (r - 64);
                arow = tile_rows(pv, tl.widx, 2 * p.nff, p.d) + (size_t)wr * row_bytes(type, p.d);
            }
        }
    }
    __device__ __forceinline__ void start(const PfParams &p, int units, int n_mb, int r) {
        u = blockIdx.x;
        seek(p, units, n_mb, r);
    }
    __device__ __forceinline__ void advance(const PfParams &p, int units, int n_mb, int nsb, int r) {
        if (++sb < nsb) return;
        sb = 0;
        if (++pass < np) return;
        u += gridDim.x;
        seek(p, units, n_mb, r);
    }
};

__global__ void __launch_bounds__(kLxThreads, 1) pf_gate_up_lx_kernel(PfParams p, const __grid_constant__ LxMaps maps) {
    extern __shared__ __align__(1024) uint8_t pf_smem[];
    LxSmem &S = *reinterpret_cast<LxSmem *>(pf_smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kLxRing; ++i) {
            mbar_init(&S.bfull[i], 1);
            mbar_init(&S.afull[i], 4);
            mbar_init(&S.opfree[i], 1);
        }
        for (int b = 0; b < kLxDBufs; ++b) {
            mbar_init(&S.dfull[b], 1);
            mbar_init(&S.dempty[b], kLxEpiWarps);
        }
        mbar_init(&S.done, kLxIssue);
        mbar_init(&S.epibar, kLxEpiWarps);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == kLxMmaWarp) tmem_alloc_warp(&S.tmem, kLxTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;
    volatile int32_t *abort = &S.abort;
    pdl_wait();
    const int nsb = p.d / QK_K, n_mb = p.nff / 64, gu_rows = 2 * p.nff;
    const int units = *p.n_tiles * n_mb * 2;

    if (warp < kLxConvWarps) {
        // ------------------------------------------------ converters: thread r = weight row r = TMEM lane r;
        // group 0 (warps 0-3) takes the even steps, group 1 (warps 4-7) the odd ones
        const int grp = warp >> 2, qd = warp & 3;
        const int r = 32 * qd + lane;
        const uint32_t ta = tmem + ((uint32_t)(32 * qd) << 16) + kLxColA;
        LxIter cur;
        cur.start(p, units, n_mb, r);
        for (int g = 0; g < grp && cur.ok; ++g) cur.advance(p, units, n_mb, nsb, r);
        for (int it = grp; cur.ok && !warp_aborted(abort); it += kLxConvGroups) {
            const int ab = it % kLxRing;
            if (tid == 0) PTRACE(0, 0, it, 0);
            if (it >= kLxRing && !lx_wait_warp(&S.opfree[ab], ((it / kLxRing) - 1) & 1, abort)) break;
            if (tid == 0) PTRACE(0, 0, it, 1);
            tc_fence_after();
            uint32_t o[32];
            if (cur.type == T_Q4_K) {
                // the step's raw blocks (and B image) have landed in ring slot ab
                if (!lx_wait_warp(&S.bfull[ab], (it / kLxRing) & 1, abort)) break;
                const uint32_t *w = reinterpret_cast<const uint32_t *>(S.raw[ab] + r * B_Q4_K);
                uint32_t scw[2], mnw[2];
                q4k_scale_words(w[1], w[2], w[3], scw, mnw);
                // per sub-block j: (sc_j, sc_j) and (-1024 sc_j, -1024 sc_j) for scale4, shared by both lanes
                __half2 s2[8], ns2[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    s2[j] = byte_h2(scw, j);
                    ns2[j] = __hmul2(s2[j], u2h(0xe400e400u));   // x -1024, exact
                }
#pragma unroll
                for (int li = 0; li < 2; ++li) {
                    const int L = lx_first_lane(cur.pass) + 4 * li;   // qs word of chunk c: 4 + 8c + L
                    const uint32_t qw[4] = {w[4 + L], w[12 + L], w[20 + L], w[28 + L]};
                    lx_a_q4k_lane(qw, s2, ns2, o + 16 * li);
                }
            } else if (cur.type == T_IQ2_S) {
                const uint8_t *blk = cur.arow + (size_t)cur.sb * B_IQ2_S;
                lx_a_iq2s_lane(blk, lx_first_lane(cur.pass), o);
                lx_a_iq2s_lane(blk, lx_first_lane(cur.pass) + 4, o + 16);
            } else {
                const uint8_t *blk = cur.arow + (size_t)cur.sb * B_IQ2_XXS;
                lx_a_iq2xxs_lane(blk, lx_first_lane(cur.pass), o);
                lx_a_iq2xxs_lane(blk, lx_first_lane(cur.pass) + 4, o + 16);
            }
            // the MMA thread waits on afull only: every converter sees the step's B image land first
            if (cur.type != T_Q4_K && !lx_wait_warp(&S.bfull[ab], (it / kLxRing) & 1, abort)) break;
            tmem_st32(ta + 32 * ab, o);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.afull[ab]);
            if (lane == 0 && grp == 0 && qd > 0) XTRACE(it, qd);
            if (tid == 0) PTRACE(0, 0, it, 2);
            for (int g = 0; g < kLxConvGroups && cur.ok; ++g) cur.advance(p, units, n_mb, nsb, r);
        }
    } else if (warp >= kLxMmaWarp && warp < kLxProdWarp) {
        // ------------------------------------------------ MMA issue: warp m takes steps m, m + kLxIssue, ...
        // in a warp-uniform loop, one elected lane issues (and commits its own MMAs). The converters
        // arrive on afull only after they saw the step's bfull, so afull alone says that both operands
        // are in place.
        const int m = warp - kLxMmaWarp;
        LxIter s;
        s.start(p, units, n_mb, -1);
        for (int g = 0; g < m && s.ok; ++g) s.advance(p, units, n_mb, nsb, -1);
        for (int it = m; s.ok && !warp_aborted(abort); it += kLxIssue) {
            const int ab = it % kLxRing, db = it % kLxDBufs;
            if (lane == 0) PTRACE(0, 1, it, 0);
            if (!lx_wait_warp(&S.afull[ab], (it / kLxRing) & 1, abort)) break;
            if (lane == 0) XTRACE(it, 12);
            if (it >= kLxDBufs && !lx_wait_warp(&S.dempty[db], ((it / kLxDBufs) - 1) & 1, abort)) break;
            if (lane == 0) XTRACE(it, 13);
            if (lane == 0) PTRACE(0, 1, it, 1);
            tc_fence_after();
            const uint32_t idesc = umma_idesc_f16(kPfM, s.N);
            const uint32_t a0 = tmem + kLxColA + 32 * ab, d0 = tmem + kLxColD + 128 * db;
            const uint32_t b0 = smem_addr(S.b[ab]);
            if (elect_one()) {
                // lane a: K = 32 into d0, lane b: K = 32 into d0 + 64
                const uint32_t sbo = kLxMainCores * 128;
                umma_f16_ts(d0, a0, umma_sdesc(b0, 128, sbo), idesc, 0);
                umma_f16_ts(d0, a0 + 8, umma_sdesc(b0 + 256, 128, sbo), idesc, 1);
                umma_f16_ts(d0 + 64, a0 + 16, umma_sdesc(b0 + 512, 128, sbo), idesc, 0);
                umma_f16_ts(d0 + 64, a0 + 24, umma_sdesc(b0 + 768, 128, sbo), idesc, 1);
                umma_commit(&S.opfree[ab]);
                umma_commit(&S.dfull[db]);
            }
            __syncwarp();
            if (lane == 0) PTRACE(0, 1, it, 2);
            for (int g = 0; g < kLxIssue && s.ok; ++g) s.advance(p, units, n_mb, nsb, -1);
        }
        // issued MMAs always complete; TMEM is freed only after them (both issuers' commits)
        if (elect_one()) umma_commit(&S.done);
        __syncwarp();
        mbar_wait(&S.done, 0);
    } else if (warp >= kLxProdWarp) {
        // ------------------------------------------------ B operand images (and Q4_K raw rows), bulk-copied
        // up to kLxRing steps ahead; warp m takes steps m, m + kLxIssue, ..., one elected lane issuing
        const int m = warp - kLxProdWarp;
        LxIter s;
        s.start(p, units, n_mb, -1);
        for (int g = 0; g < m && s.ok; ++g) s.advance(p, units, n_mb, nsb, -1);
        for (int it = m; s.ok && !warp_aborted(abort); it += kLxIssue) {
            const int bs = it % kLxRing;
            if (it >= kLxRing && !lx_wait_warp(&S.opfree[bs], ((it / kLxRing) - 1) & 1, abort)) break;
            const uint32_t bytes = (uint32_t)(s.N / 8) * kLxMainCores * 128;
            const bool q4 = s.type == T_Q4_K;
            if (elect_one()) {
                mbar_expect_tx(&S.bfull[bs], bytes + (q4 ? (uint32_t)kLxRawBytes : 0u));
                bulk_g2s(S.b[bs],
                         p.bimg + (size_t)s.ti * lx_tile_bytes(nsb) + lx_image_off(nsb, s.pass, s.sb) +
                             (size_t)(8 * s.nh) * kLxMainCores * 128,
                         bytes, &S.bfull[bs]);
                if (q4) {   // rows [64 mb, +64) and [n_ff + 64 mb, +64) of the entry, bytes [144 sb, +144)
                    const CUtensorMap *map = s.tl.cls ? &maps.gu[1] : &maps.gu[0];
                    const int y0 = s.tl.widx * gu_rows + 64 * s.mb;
                    tma_load_2d(S.raw[bs], map, s.sb * B_Q4_K, y0, &S.bfull[bs]);
                    tma_load_2d(S.raw[bs] + 64 * B_Q4_K, map, s.sb * B_Q4_K, y0 + p.nff, &S.bfull[bs]);
                }
                XTRACE(it, 0);
            }
            __syncwarp();
            for (int g = 0; g < kLxIssue && s.ok; ++g) s.advance(p, units, n_mb, nsb, -1);
        }
    } else {
        // ------------------------------------------------ epilogue: the lanes' f32 chains
        const int ew = warp - kLxEpiWarp0, et = tid - kLxEpiWarp0 * 32;
        const int q = warp & 3, ch = ew >> 2;
        const int r = 32 * q + lane, col0 = kLxEpiCols * ch;
        const uint32_t tl_lane = tmem + ((uint32_t)(32 * q) << 16);
        int it = 0;
        uint32_t eph = 0;
        LxIter s;
        s.start(p, units, n_mb, r);
        while (s.ok && !warp_aborted(abort)) {
            const int ti = s.ti, nh = s.nh, np = s.np, nc = s.nc, type = s.type;
            const PfTile tl = s.tl;
            const uint8_t *arow = s.arow;
            const int wr = r < 64 ? 64 * s.mb + r : p.nff + 64 * s.mb + (r - 64);
            for (int i = et; i < nsb * kLxN; i += kLxEpiWarps * 32) {
                const int sb = i / kLxN, j = i - sb * kLxN;
                S.dxs[sb][j] = p.dxt[((size_t)ti * nsb + sb) * kPfN + 64 * nh + j];
            }
            if (ch == 0) {   // the row's d_w per super-block (the first fp16 of every block type here)
                const int bsz = type == T_Q4_K ? B_Q4_K : type == T_IQ2_S ? B_IQ2_S : B_IQ2_XXS;
                for (int sb = 0; sb < nsb; ++sb)
                    S.xdt[sb][r] = h2f(__ldg(reinterpret_cast<const uint16_t *>(arow + (size_t)sb * bsz)));
            }
            if (!epi_barrier(&S.epibar, eph, abort)) break;
            const bool live = col0 < s.N;   // this warp's columns hold MMA output
            bool ok = true;
            for (int pass = 0; pass < np && ok; ++pass) {
                uint64_t accA[kLxEpiCols / 2], accB[kLxEpiCols / 2];
#pragma unroll
                for (int i = 0; i < kLxEpiCols / 2; ++i) { accA[i] = 0ull; accB[i] = 0ull; }
                for (int sb = 0; sb < nsb; ++sb, ++it) {
                    const int db = it % kLxDBufs;
                    if (et == 0) PTRACE(0, 2, it, 0);
                    if (!lx_wait_warp(&S.dfull[db], (it / kLxDBufs) & 1, abort)) { ok = false; break; }
                    if (et == 0) PTRACE(0, 2, it, 1);
                    tc_fence_after();
                    if (live) {
                        const float xs = S.xdt[sb][r];   // d_w
                        const uint64_t xs2 = f2pack(xs, xs);
                        const uint32_t dcol = tl_lane + kLxColD + 128 * db + col0;
                        const float4 *yd = reinterpret_cast<const float4 *>(&S.dxs[sb][col0]);
                        // the warp's 16 columns of both lanes in one TMEM round trip
                        static_assert(kLxEpiCols == 16, "one x16 load per lane");
                        uint32_t sa[16], sbv[16];
                        tmem_ld16x2u(dcol, dcol + 64, sa, sbv);
                        if (et == 0) XTRACE(it, 15);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float4 y4 = yd[i];
                            // d = d_x * d_w rounded to f32
                            const uint64_t d01 = mul2(f2pack(y4.x, y4.y), xs2), d23 = mul2(f2pack(y4.z, y4.w), xs2);
                            const int k0 = 2 * i;
                            accA[k0] = fma2(d01, f2pack(__uint_as_float(sa[4 * i]), __uint_as_float(sa[4 * i + 1])), accA[k0]);
                            accB[k0] = fma2(d01, f2pack(__uint_as_float(sbv[4 * i]), __uint_as_float(sbv[4 * i + 1])), accB[k0]);
                            accA[k0 + 1] = fma2(d23, f2pack(__uint_as_float(sa[4 * i + 2]), __uint_as_float(sa[4 * i + 3])),
                                                accA[k0 + 1]);
                            accB[k0 + 1] = fma2(d23, f2pack(__uint_as_float(sbv[4 * i + 2]), __uint_as_float(sbv[4 * i + 3])),
                                                accB[k0 + 1]);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.dempty[db]);
                    if (lane == 0) XTRACE(it, 4 + ew);
                    if (et == 0) PTRACE(0, 2, it, 2);
                }
                if (!ok || !live) continue;
                // fold the finished pass in the reference's reduction order (aL = the pass's lane pair
                // sum a_L + a_{L+4}):  pass 0: Ha = a0;  1: Ha = a0 + a2 = c0;  2: Hb = a1;
                // 3: h = c0 + (a1 + a3), then Q4_K: h + M (M from pf_q4k_min_kernel, already in hbuf),
                // IQ2_S / IQ2_XXS: h x 1/8
                float t[kLxEpiCols];
#pragma unroll
                for (int i = 0; i < kLxEpiCols / 2; ++i) {
                    const float2 v = f2unpack(add2(accA[i], accB[i]));
                    t[2 * i] = v.x;
                    t[2 * i + 1] = v.y;
                }
                float(*ha)[kPfM] = S.held[0] + col0;
                float(*hb)[kPfM] = S.held[1] + col0;
                if (pass == 0 || pass == 2) {
#pragma unroll
                    for (int i = 0; i < kLxEpiCols; ++i) (pass == 0 ? ha : hb)[i][r] = t[i];
                    continue;
                }
#pragma unroll
                for (int i = 0; i < kLxEpiCols; ++i) t[i] = __fadd_rn((pass == 1 ? ha : hb)[i][r], t[i]);
                if (pass == 1) {
#pragma unroll
                    for (int i = 0; i < kLxEpiCols; ++i) ha[i][r] = t[i];
                    continue;
                }
                // pass 3: Ha = c0, t = c1
#pragma unroll
                for (int i = 0; i < kLxEpiCols; ++i) t[i] = __fadd_rn(ha[i][r], t[i]);
                // the unit's rows for this warp's pairs, f32, slot order ([slot][2 n_ff])
                float *hbp = p.hbuf + (size_t)(tl.slot0 + 64 * nh + col0) * gu_rows + wr;
                if (type == T_Q4_K) {
#pragma unroll
                    for (int i = 0; i < kLxEpiCols; ++i)
                        if (col0 + i < nc) t[i] = __fadd_rn(t[i], hbp[(size_t)i * gu_rows]);
                } else {
#pragma unroll
                    for (int i = 0; i < kLxEpiCols; ++i) t[i] = __fmul_rn(0.125f, t[i]);
                }
#pragma unroll
                for (int i = 0; i < kLxEpiCols; ++i)
                    if (col0 + i < nc) hbp[(size_t)i * gu_rows] = t[i];
            }
            if (!ok || !epi_barrier(&S.epibar, eph, abort)) break;
            s.u += gridDim.x;
            s.seek(p, units, n_mb, r);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kLxMmaWarp) {
        tc_fence_after();
        tmem_dealloc_warp(tmem, kLxTmemCols);
    }
}

}  // namespace moeb
