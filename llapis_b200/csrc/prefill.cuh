// Prefill path of the MoE-FFN layer: the same layer as the fused decode kernel, for batches large
// enough that every routed expert sees many tokens. Ten kernels chained with programmatic
// dependent launch:
//
//   pf_router_kernel     : router logits, f32 GEMM (ggml mul_mat of ffn_gate_inp, gemma4.cpp:403)
//   pf_topk_kernel       : softmax -> top-k (value desc, index asc) -> normalised weights
//                          (llama-graph.cpp:1553-1648), one warp per token
//   pf_dispatch_kernel   : histogram, exclusive scan and stable permutation of the routed pairs
//                          (ggml-cpu.c:1613-1626 grouping; mmid.cu:28 on the GPU) plus the per-expert
//                          tile list the grouped GEMMs walk
//   pf_actq_kernel       : Q8_K quantisation of every token (quantize_row_q8_K, x86/quants.c:505);
//                          pf_actq_norm_kernel with the block norms, pf_unpack_q8k_kernel for rows
//                          that arrive already quantised
//   pf_gather_lx_kernel  : per expert tile, the tokens' Q8_K values as fp16 operand images in the
//                          reference's lane order (gateup_lx.cuh)
//   pf_q4k_min_kernel    : the Q4_K min term of every (row, pair) (gateup_lx.cuh)
//   pf_gate_up_lx_kernel : tcgen05 grouped GEMM, gate_up of every tile in the reference's float
//                          order (gateup_lx.cuh), f32 rows in slot order
//   pf_geglu_kernel      : GeGLU (fp16-table GELU, vec.h:1414) and Q8_0 quantisation of its output
//                          (x86/quants.c:302) into the down kernel's fp16 operand images
//   pf_down_kernel       : tcgen05 grouped GEMM, down projection, per-expert down scale
//   pf_combine_kernel    : out[t] = sum_j w[t,j] * y[t,j] in j order (llama-graph.cpp:1814-1848)
//
// Integer-exact tensor-core formulation. ggml-cpu computes the expert matmuls as integer block
// dot products scaled per block (ggml_vec_dot_q4_K_q8_K, x86/quants.c:1900; _iq2_s_q8_K :2937;
// _q5_0_q8_0; _iq4_nl_q8_0). The MMAs here reproduce the integer sums exactly with kind::f16
// operands that are small integers (exactly representable in fp16) and fp32 accumulation, and
// apply the per-block float scales in the epilogue ("promotion"):
//   gate_up      : gateup_lx.cuh (one accumulator per reference lane, the lanes' f32 chains in the
//                  reference's order).
//   down Q5_0    : A = q - 16; B = d_x * q8 (the Q8_0 GeGLU output, dequantised) split exactly
//                  into fp16 hi + lo, two MMAs per K step; promoted per 32-block with d_w.
//   down IQ4_NL  : A = kvalues_iq4nl[q], B as for Q5_0.
// Converter warps build the fp16 weight (A) tiles in shared memory; the activation (B) tiles are
// fp16 images in HBM (written by pf_geglu_kernel) fetched with one bulk copy per stage. The A tiles
// use the canonical no-swizzle K-major layout (8-row x 16-byte core matrices), one thread issues
// the MMAs, accumulators live in TMEM (quadruple-buffered so the MMAs of the next block overlap the
// promotion of the last), and epilogue warps read them back with tcgen05.ld.
#pragma once

namespace moeb {

// ---------------------------------------------------------------- tcgen05 / UMMA wrappers
// Shared-memory matrix descriptor (sm100 UMMA): start address, leading byte offset (distance of
// the next core matrix along K), stride byte offset (distance of the next 8-row group), version 1,
// no swizzle.
__device__ __forceinline__ uint64_t umma_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D, shape M x N.
__device__ __forceinline__ uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}
// arrive on `bar` once every MMA this thread issued so far has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_alloc_warp(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_warp(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

#define MOEB_R16(a) "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), \
    "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15])
#define MOEB_RW16(a) "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), \
    "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15])
#define MOEB_LD16 "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"

// 16 consecutive accumulator columns of this thread's TMEM lane (the wait is tied to the
// registers so no use of them can be scheduled before it)
__device__ __forceinline__ void tmem_ld16(uint32_t ta, float (&va)[16]) {
    uint32_t a[16];
    asm volatile(MOEB_LD16 : MOEB_R16(a) : "r"(ta));
    asm volatile("tcgen05.wait::ld.sync.aligned;" : MOEB_RW16(a)::"memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) va[i] = __uint_as_float(a[i]);
}
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, float (&va)[16], float (&vb)[16]) {
    uint32_t a[16], b[16];
    asm volatile(MOEB_LD16 : MOEB_R16(a) : "r"(ta));
    asm volatile(MOEB_LD16 : MOEB_R16(b) : "r"(tb));
    asm volatile("tcgen05.wait::ld.sync.aligned;" : MOEB_RW16(a), MOEB_RW16(b)::"memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) { va[i] = __uint_as_float(a[i]); vb[i] = __uint_as_float(b[i]); }
}

// Instrumented builds only (-DMOEB_TRACE): SM-clock stamps of CTA 0's converter warp 0, MMA thread
// and first epilogue warp, per pipeline step.
#ifdef MOEB_TRACE
__device__ unsigned long long g_ptrace[2][3][256][3];
__device__ unsigned long long g_utrace[32][16];
__device__ unsigned long long g_xtrace[256][16];
#define XTRACE(idx, f) \
    if (blockIdx.x == 0 && (idx) < 256) g_xtrace[idx][f] = clock64();
#define PTRACE(k, role, idx, f) \
    if (blockIdx.x == 0 && (idx) < 256) g_ptrace[k][role][idx][f] = clock64();
#define UTRACE(u, f) \
    if (blockIdx.x == 0 && (u) < 32) g_utrace[u][f] = clock64();
#else
#define PTRACE(k, role, idx, f)
#define UTRACE(u, f)
#define XTRACE(idx, f)
#endif

// ---------------------------------------------------------------- shapes of the tensor-core kernels
constexpr int kPfN = kPrefillTile;    // routed pairs per expert tile = MMA N (accumulator columns)
constexpr int kPfM = 128;             // weight rows per work unit = MMA M (TMEM lanes)
constexpr int kPfConvWarps = 4;       // thread i builds A row i (a weight row) and B row i (a pair)
constexpr int kPfMmaWarp = kPfConvWarps;
constexpr int kPfEpiWarp0 = kPfConvWarps + 1;
// down: a stage is two 32-blocks (8 core columns); four accumulator buffers of 128 columns
constexpr int kDnKc = 8;
constexpr int kDnTileBytes = kPfM * kDnKc * 16;
constexpr int kDnStages = 4;
// down: 16 epilogue warps, four per TMEM lane quadrant, 32 columns each (one TMEM round trip per
// 32-block); 21 warps leave 80 registers a thread
constexpr int kDnEpiWarps = 16;
constexpr int kDnThreads = (kPfConvWarps + 1 + kDnEpiWarps) * 32;
constexpr int kDnAccBufs = 4;
static_assert(kPfN == 128 && kPfM == 128, "TMEM budget below assumes 128 x 128 tiles");

// byte offset of core row (r, c) of a canonical K-major tile with kc core columns per 8-row group
__device__ __forceinline__ uint32_t canon_off(int r, int c, int kc) {
    return (uint32_t)((((r >> 3) * kc + c) << 7) + ((r & 7) << 4));
}

struct DnSmem {
    uint8_t a[kDnStages][kDnTileBytes];
    uint8_t b[kDnStages][2 * kDnTileBytes];   // hi and lo halves of dx * q8
    uint64_t full[kDnStages], empty[kDnStages], accfull[kDnAccBufs], accempty[kDnAccBufs], done, epibar;
    uint32_t tmem;
    int32_t abort;
};

// Bounded mbarrier wait that also gives up once another role of the CTA has given up.
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int32_t *abort) {
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *abort) return false;
    }
    atomicOr(&g_error, ERR_MBAR_TIMEOUT);
    *abort = 1;
    return false;
}
// the abort flag as one value for the whole warp (loop conditions must not split a warp)
__device__ __forceinline__ bool warp_aborted(volatile int32_t *abort) { return __any_sync(0xffffffffu, *abort != 0); }
// The same wait taken by every lane of a warp, with one outcome for the whole warp (so that a
// warp never splits before a .sync.aligned instruction).
__device__ __forceinline__ bool pf_wait_warp(uint64_t *bar, uint32_t parity, volatile int32_t *abort) {
    return __all_sync(0xffffffffu, pf_wait(bar, parity, abort));
}
// Barrier of the epilogue warps on an mbarrier (count: the epilogue warps): bounded, unlike bar.sync, so a
// warp that gave up cannot leave the others waiting for good.
__device__ __forceinline__ bool epi_barrier(uint64_t *bar, uint32_t &phase, volatile int32_t *abort) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const bool ok = pf_wait_warp(bar, phase & 1u, abort);
    ++phase;
    return ok;
}

// ---------------------------------------------------------------- fp16 operand builders
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
// four small unsigned byte values (one per byte of t) times s, as two fp16 pairs. 0x64XX is the
// fp16 1024 + XX, so (1024 + v) * s - 1024 * s = v * s, exact while v * s < 2048 and
// (1024 + v) * s < 65504.
__device__ __forceinline__ void scale4(uint32_t t, __half2 s2, __half2 ns2, uint32_t &o01, uint32_t &o23) {
    o01 = h2u(__hfma2(u2h(__byte_perm(t, 0x64646464u, 0x5140)), s2, ns2));
    o23 = h2u(__hfma2(u2h(__byte_perm(t, 0x64646464u, 0x5342)), s2, ns2));
}
// four signed bytes as two fp16 pairs (exact): (1024 + (v ^ 0x80)) - 1152 = v
__device__ __forceinline__ void s8x4_h(uint32_t w, uint32_t &o01, uint32_t &o23) {
    const uint32_t u = w ^ 0x80808080u;
    const __half2 off = u2h(0xe480e480u);   // (-1152, -1152)
    o01 = h2u(__hadd2(u2h(__byte_perm(u, 0x64646464u, 0x5140)), off));
    o23 = h2u(__hadd2(u2h(__byte_perm(u, 0x64646464u, 0x5342)), off));
}
// four unsigned bytes < 32 minus 16, as two fp16 pairs (exact): (1024 + u) - 1040
__device__ __forceinline__ void u5x4_h(uint32_t t, uint32_t &o01, uint32_t &o23) {
    const __half2 off = u2h(0xe410e410u);   // (-1040, -1040)
    o01 = h2u(__hadd2(u2h(__byte_perm(t, 0x64646464u, 0x5140)), off));
    o23 = h2u(__hadd2(u2h(__byte_perm(t, 0x64646464u, 0x5342)), off));
}
__device__ __forceinline__ uint32_t pack_h2i(int a, int b) {
    return h2u(__floats2half2_rn((float)a, (float)b));   // exact for the small integers used here
}
__device__ __forceinline__ void sts128(uint8_t *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<uint4 *>(p) = make_uint4(a, b, c, d);
}


// Raw bytes of one down stage: two Q5_0 blocks (11 words) or two IQ4_NL blocks (9 words) of a
// weight row, 4-byte aligned (44- and 36-byte stages of 484- and 396-byte rows)
struct DnARaw {
    uint32_t w[11];
};
__device__ __forceinline__ void dn_a_load(const uint8_t *src, bool q5, DnARaw &a) {
    const unsigned int *w = reinterpret_cast<const unsigned int *>(src);
#pragma unroll
    for (int i = 0; i < 9; ++i) a.w[i] = __ldg(w + i);
    a.w[9] = q5 ? __ldg(w + 9) : 0u;
    a.w[10] = q5 ? __ldg(w + 10) : 0u;
}

// A rows of one down stage, Q5_0 (dequantize_row_q5_0, ggml-quants.c:442): q - 16 with
// q = nibble | high bit << 4
__device__ __forceinline__ void dn_a_q5_0(const DnARaw &a, uint8_t *tile, int r) {
#pragma unroll
    for (int bi = 0; bi < 2; ++bi) {
        uint32_t qh, qs[4];
        if (bi == 0) {   // d bytes 0-1, qh 2-5, qs 6-21
            qh = __funnelshift_r(a.w[0], a.w[1], 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) qs[i] = __funnelshift_r(a.w[1 + i], a.w[2 + i], 16);
        } else {         // d bytes 22-23, qh 24-27, qs 28-43
            qh = a.w[6];
#pragma unroll
            for (int i = 0; i < 4; ++i) qs[i] = a.w[7 + i];
        }
#pragma unroll
        for (int cq = 0; cq < 4; ++cq) {
            // values 8cq .. 8cq+7: low nibbles of qs bytes for cq < 2, high nibbles of bytes 8(cq-2).. for cq >= 2
            const uint32_t a0 = cq < 2 ? qs[2 * cq] : qs[2 * (cq - 2)] >> 4;
            const uint32_t a1 = cq < 2 ? qs[2 * cq + 1] : qs[2 * (cq - 2) + 1] >> 4;
            const uint32_t hb = (qh >> (8 * cq)) & 0xffu;
            const uint32_t t0 = (a0 & 0x0f0f0f0fu) | ((((hb & 0xfu) * 0x00204081u) & 0x01010101u) << 4);
            const uint32_t t1 = (a1 & 0x0f0f0f0fu) | ((((hb >> 4) * 0x00204081u) & 0x01010101u) << 4);
            uint32_t o0, o1, o2, o3;
            u5x4_h(t0, o0, o1);
            u5x4_h(t1, o2, o3);
            sts128(tile + canon_off(r, 4 * bi + cq, kDnKc), o0, o1, o2, o3);
        }
    }
}

// A rows of one down stage, IQ4_NL (dequantize_row_iq4_nl, ggml-quants.c:2653): kvalues[q]
__device__ __forceinline__ void dn_a_iq4nl(const DnARaw &a, const uint32_t (&kv)[4], uint8_t *tile, int r) {
#pragma unroll
    for (int bi = 0; bi < 2; ++bi) {
        uint32_t qs[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qs[i] = bi == 0 ? __funnelshift_r(a.w[i], a.w[i + 1], 16) : a.w[5 + i];
#pragma unroll
        for (int cq = 0; cq < 4; ++cq) {
            const uint32_t a0 = cq < 2 ? qs[2 * cq] : qs[2 * (cq - 2)] >> 4;
            const uint32_t a1 = cq < 2 ? qs[2 * cq + 1] : qs[2 * (cq - 2) + 1] >> 4;
            uint32_t o0, o1, o2, o3;
            s8x4_h((uint32_t)iq4nl_lookup4(a0, kv[0], kv[1], kv[2], kv[3]), o0, o1);
            s8x4_h((uint32_t)iq4nl_lookup4(a1, kv[0], kv[1], kv[2], kv[3]), o2, o3);
            sts128(tile + canon_off(r, 4 * bi + cq, kDnKc), o0, o1, o2, o3);
        }
    }
}


struct PfParams {
    int32_t T, E, d, k, nff;
    PoolView gu[2], dn[2];            // [0] hot, [1] cold
    const int32_t *perm;              // [P] slot -> pair (t*k + j)
    const PfTile *tiles;
    const int32_t *n_tiles;
    const int8_t *xq8;                // [T][d] Q8_K values
    const float *xd;                  // [T][d/256] Q8_K scales
    const int16_t *xbs;               // [T][d/256][16] Q8_K bsums
    uint8_t *bimg;                    // gate_up B operand images, [tile][pass][sb][kLxImgMain] (or the mid path's)
    float *dxt;                       // [tile][sb][128] Q8_K scale of each tile row
    uint32_t *bst;                    // [tile][sb][128][8] Q8_K bsums of each tile row, fp16 pairs
    float *hbuf;                      // [slot][2 n_ff] gate_up outputs, f32
    uint8_t *dimg;                    // down B operand images, [tile][stage][kPfDnImageBytes]

    float *h;                         // optional [P pairs][2 nff] gate_up outputs
    float *y;                         // [P slots][d] down outputs (scaled)
};

__device__ __forceinline__ const uint8_t *tile_rows(const PoolView &pv, int widx, int rows, int d_in) {
    return pool_entry(pv, widx, rows, d_in);
}

// ---------------------------------------------------------------- down grouped GEMM
// Work unit (tile, mb): the pairs of one expert tile against down rows [128 mb, 128 mb + 128).
__global__ void __launch_bounds__(kDnThreads, 1) pf_down_kernel(PfParams p) {
    extern __shared__ __align__(1024) uint8_t pf_smem[];
    DnSmem &S = *reinterpret_cast<DnSmem *>(pf_smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kDnStages; ++s) { mbar_init(&S.full[s], kPfConvWarps + 1); mbar_init(&S.empty[s], 1); }
        for (int b = 0; b < kDnAccBufs; ++b) { mbar_init(&S.accfull[b], 1); mbar_init(&S.accempty[b], kDnEpiWarps); }
        mbar_init(&S.done, 1);
        mbar_init(&S.epibar, kDnEpiWarps);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == kPfMmaWarp) tmem_alloc_warp(&S.tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;
    volatile int32_t *abort = &S.abort;
    pdl_wait();
    const int n_mb = p.d / kPfM, nblk = p.nff / QK32, nst = nblk / 2;
    const int units = *p.n_tiles * n_mb;

    if (warp < kPfConvWarps) {
        uint32_t kv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            kv[i] = (uint32_t)(uint8_t)g_iq4nl[4 * i] | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 1] << 8) |
                    ((uint32_t)(uint8_t)g_iq4nl[4 * i + 2] << 16) | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 3] << 24);
        int it = 0;
        DnARaw ar0, ar1;
        for (int u = blockIdx.x; u < units && !warp_aborted(abort); u += gridDim.x) {
            const int ti = u / n_mb, mb = u - ti * n_mb;
            const PfTile tl = p.tiles[ti];
            const PoolView &pv = p.dn[tl.cls];
            const bool q5 = pv.type == T_Q5_0;
            const int rb = (int)row_bytes(pv.type, p.nff);
            const int r = tid;
            const uint8_t *arow = tile_rows(pv, tl.widx, p.d, p.nff) + (size_t)(kPfM * mb + r) * rb;
            const uint32_t bbytes = (uint32_t)(((tl.n + 15) & ~15) / 8) * (kDnKc * 128);
            const uint8_t *bsrc = p.dimg + (size_t)ti * nst * 2 * kPfDnImageBytes;
            const int sbytes = q5 ? 2 * B_Q5_0 : 2 * B_IQ4_NL;
            dn_a_load(arow, q5, ar0);
            if (nst > 1) dn_a_load(arow + sbytes, q5, ar1);
            for (int st0 = 0; st0 < nst; st0 += 2) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int st = st0 + e;
                    if (st >= nst) break;
                    const int s = it % kDnStages;
                    if (tid == 0) PTRACE(1, 0, it, 0);
                    if (it >= kDnStages && !pf_wait_warp(&S.empty[s], ((it / kDnStages) - 1) & 1, abort)) { st0 = nst; break; }
                    if (tid == 0) {
                        PTRACE(1, 0, it, 1);
                        mbar_expect_tx(&S.full[s], 2 * bbytes);
                        bulk_g2s(S.b[s], bsrc + (size_t)st * 2 * kPfDnImageBytes, bbytes, &S.full[s]);
                        bulk_g2s(S.b[s] + kDnTileBytes, bsrc + (size_t)st * 2 * kPfDnImageBytes + kPfDnImageBytes, bbytes,
                                 &S.full[s]);
                    }
                    DnARaw &ar = e == 0 ? ar0 : ar1;
                    if (q5) dn_a_q5_0(ar, S.a[s], r);
                    else dn_a_iq4nl(ar, kv, S.a[s], r);
                    if (st + 2 < nst) dn_a_load(arow + (st + 2) * sbytes, q5, ar);   // two stages ahead
                    if (tid == 0) PTRACE(1, 0, it, 2);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.full[s]);
                    ++it;
                }
            }
        }
    } else if (warp == kPfMmaWarp) {
        if (lane == 0) {
            int it = 0, ac = 0;
            const uint32_t sbo = kDnKc * 128;
            for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x) {
                const PfTile tl = p.tiles[u / n_mb];
                const int N = (tl.n + 15) & ~15;
                const uint32_t idesc = umma_idesc_f16(kPfM, N);
                for (int st = 0; st < nst && !*abort; ++st, ++it) {
                    const int s = it % kDnStages;
                    PTRACE(1, 1, it, 0);
                    if (!pf_wait(&S.full[s], (it / kDnStages) & 1, abort)) break;
                    PTRACE(1, 1, it, 1);
                    tc_fence_after();
                    const uint32_t a0 = smem_addr(S.a[s]), b0 = smem_addr(S.b[s]);
                    for (int bi = 0; bi < 2; ++bi, ++ac) {
                        const int b = ac % kDnAccBufs;
                        if (ac >= kDnAccBufs && !pf_wait(&S.accempty[b], ((ac / kDnAccBufs) - 1) & 1, abort)) break;
                        tc_fence_after();
                        const uint32_t dt = tmem + (uint32_t)(b * 128);
#pragma unroll
                        for (int ks = 0; ks < 2; ++ks) {
                            const uint32_t off = (uint32_t)((4 * bi + 2 * ks) * 128);
                            const uint64_t da = umma_sdesc(a0 + off, 128, sbo);
                            umma_f16(dt, da, umma_sdesc(b0 + off, 128, sbo), idesc, ks);                    // dx*q8 hi
                            umma_f16(dt, da, umma_sdesc(b0 + kDnTileBytes + off, 128, sbo), idesc, 1u);      // dx*q8 lo
                        }
                        umma_commit(&S.accfull[b]);
                    }
                    umma_commit(&S.empty[s]);
                    PTRACE(1, 1, it, 2);
                }
            }
            umma_commit(&S.done);
            mbar_wait(&S.done, 0);   // issued MMAs always complete; TMEM is freed only after them
        }
        __syncwarp();
    } else {
        // epilogue: warp -> (lane quadrant q, column quarter cq); promotion per 32-block by the
        // row's d_w (the activation scale is already in the operand)
        const int ew = warp - kPfEpiWarp0;
        const int q = warp & 3, cq = ew >> 2;
        const int r = 32 * q + lane, c0 = 32 * cq;
        int ac = 0;
        uint32_t eph = 0;
        for (int u = blockIdx.x; u < units && !warp_aborted(abort); u += gridDim.x) {
            const int ti = u / n_mb, mb = u - ti * n_mb;
            const PfTile tl = p.tiles[ti];
            const PoolView &pv = p.dn[tl.cls];
            const int bsz = pv.type == T_Q5_0 ? B_Q5_0 : B_IQ4_NL;
            const int rb = (int)row_bytes(pv.type, p.nff);
            const int N = (tl.n + 15) & ~15;
            const uint16_t *dwp = reinterpret_cast<const uint16_t *>(tile_rows(pv, tl.widx, p.d, p.nff) +
                                                                     (size_t)(kPfM * mb + r) * rb);
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.f;
            uint16_t dw_next = __ldg(reinterpret_cast<const unsigned short *>(dwp));
            for (int bk = 0; bk < nblk; ++bk, ++ac) {
                const float dw = h2f(dw_next);
                if (bk + 1 < nblk) dw_next = __ldg(reinterpret_cast<const unsigned short *>(dwp) + (bk + 1) * (bsz / 2));
                const int b = ac % kDnAccBufs;
                if (ew == 0 && lane == 0) PTRACE(1, 2, ac, 0);
                if (!pf_wait_warp(&S.accfull[b], (ac / kDnAccBufs) & 1, abort)) break;
                if (ew == 0 && lane == 0) PTRACE(1, 2, ac, 1);
                tc_fence_after();
                const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * 128 + c0);
                if (c0 < N) {
                    float v[32];
                    if (c0 + 16 < N) {
                        tmem_ld16x2(tb, tb + 16, *reinterpret_cast<float(*)[16]>(&v[0]), *reinterpret_cast<float(*)[16]>(&v[16]));
#pragma unroll
                        for (int i = 0; i < 32; ++i) acc[i] = fmaf(dw, v[i], acc[i]);
                    } else {
                        tmem_ld16(tb, *reinterpret_cast<float(*)[16]>(&v[0]));
#pragma unroll
                        for (int i = 0; i < 16; ++i) acc[i] = fmaf(dw, v[i], acc[i]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.accempty[b]);
                if (ew == 0 && lane == 0) PTRACE(1, 2, ac, 2);
            }
            if (warp_aborted(abort)) break;
            const float sc = pv.scale ? pv.scale[tl.widx] : 1.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int col = c0 + i;
                if (col < tl.n) p.y[(size_t)(tl.slot0 + col) * p.d + kPfM * mb + r] = pv.scale ? __fmul_rn(acc[i], sc) : acc[i];
            }
            if (!epi_barrier(&S.epibar, eph, abort)) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPfMmaWarp) {
        tc_fence_after();
        tmem_dealloc_warp(tmem, 512);
    }
}

// ---------------------------------------------------------------- GeGLU + Q8_0 -> down operand images
// CTA per (tile, 32-output block); warp per tile row (pair), lane = output: a = geglu1(g, u) with
// ggml-cpu's fp16-table GELU (vec.h:1414), Q8_0 of the 32 values (AVX2 quantize_row_q8_0
// semantics), written as fp16 into the tile's down operand image, the scale into the tile's
// per-row table. A kernel of its own: the table lookups are random, and here the table stays
// in L2 instead of being evicted by the weight stream of the GEMMs.
__global__ void __launch_bounds__(256) pf_geglu_kernel(PfParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const int ti = blockIdx.x, blk = blockIdx.y;
    if (ti >= *p.n_tiles) return;
    const PfTile tl = p.tiles[ti];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nff = p.nff;
    // lane (row rr, quarter qk): 8 consecutive values K = 32 blk + 8 qk .. + 7 of the block for pair
    // row rr of the warp's 8 rows; the block's Q8_0 amax is a max over the 4 lanes of the row, and
    // every lane writes whole 16-byte core-matrix rows of the hi and lo operand images
    const int rr = lane >> 2, qk = lane & 3;
    const int st = blk >> 1, kcol = 4 * (blk & 1) + qk;
    uint8_t *dimg = p.dimg + ((size_t)ti * (nff / 64) + st) * 2 * kPfDnImageBytes;
    for (int c = warp * 8 + rr; c - rr < tl.n; c += 64) {   // warp-uniform bound: the row block starts in the tile
        const bool valid = c < tl.n;
        float g[8], u[8];
        const float *hr = p.hbuf + (size_t)(tl.slot0 + (valid ? c : 0)) * 2 * nff + 32 * blk + 8 * qk;
        const float4 g0 = *reinterpret_cast<const float4 *>(hr), g1 = *reinterpret_cast<const float4 *>(hr + 4);
        const float4 u0 = *reinterpret_cast<const float4 *>(hr + nff), u1 = *reinterpret_cast<const float4 *>(hr + nff + 4);
        g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w; g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
        u[0] = u0.x; u[1] = u0.y; u[2] = u0.z; u[3] = u0.w; u[4] = u1.x; u[5] = u1.y; u[6] = u1.z; u[7] = u1.w;
        uint16_t tv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) tv[j] = g_gelu_f16[f2h_rn(g[j])];
        float a[8], m = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            a[j] = g[j] <= -10.0f ? 0.0f : (g[j] >= 10.0f ? __fmul_rn(g[j], u[j]) : __fmul_rn(h2f(tv[j]), u[j]));
            m = fmaxf(m, fabsf(a[j]));
        }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        if (!valid) continue;
        const float dd = h2f(f2h_rn(__fdiv_rn(m, 127.f)));
        const float id = m != 0.f ? __fdiv_rn(127.f, m) : 0.f;
        // the down operand is dx * q8 (exact in f32: an fp16 scale times a 7-bit integer), split into
        // fp16 hi + lo, both exact: the value and its parts are multiples of 2^-24 with at most 18
        // significant bits
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const float v0 = __fmul_rn(dd, (float)__float2int_rn(__fmul_rn(a[j], id)));
            const float v1 = __fmul_rn(dd, (float)__float2int_rn(__fmul_rn(a[j + 1], id)));
            if (fabsf(v0) > 65504.f || fabsf(v1) > 65504.f) atomicOr(&g_error, ERR_RANGE);
            const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
            const __half l0 = __float2half_rn(__fsub_rn(v0, __half2float(h0)));
            const __half l1 = __float2half_rn(__fsub_rn(v1, __half2float(h1)));
            hw[j / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lw[j / 2] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        const uint32_t off = canon_off(c, kcol, kDnKc);
        *reinterpret_cast<uint4 *>(dimg + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4 *>(dimg + kPfDnImageBytes + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        if (p.h) {
            float *hp = p.h + (size_t)p.perm[tl.slot0 + c] * 2 * nff + 32 * blk + 8 * qk;
            *reinterpret_cast<float4 *>(hp) = g0;
            *reinterpret_cast<float4 *>(hp + 4) = g1;
            *reinterpret_cast<float4 *>(hp + nff) = u0;
            *reinterpret_cast<float4 *>(hp + nff + 4) = u1;
        }
    }
}

// ---------------------------------------------------------------- router, routing, dispatch, act quant
// Router logits, f32 SIMT GEMM (no tensor cores: the logits decide the routing, so they keep f32
// products; the reference's ggml mul_mat is f32 too). CTA: 64 tokens x 128 experts x one quarter
// of K, 256 threads of 8 experts x 4 tokens; K in chunks of 32 staged k-major in shared memory,
// the next chunk prefetched into registers. The nsplit K parts land in part[nsplit][T][E] and
// the top-k kernel adds them in order (deterministic); with nsplit = 1, part may be the logits
// buffer itself (the top-k kernel completes it in place).
constexpr int kRtTok = 64, kRtExp = 128, kRtK = 32, kRtSplit = 4;
// With the Gemma-4 block norms (nscale given) the x values become the router input
// rms_norm(x) / sqrt(d) * router_scale as they are staged.
__global__ void __launch_bounds__(256) pf_router_kernel(const float *W, const float *x, float *part, int T, int E,
                                                        int d, int nsplit, const float *nscale, const float *rscale) {
    __shared__ __align__(16) float ws[kRtK][kRtExp];
    __shared__ __align__(16) float xs[kRtK][kRtTok];
    pdl_wait();
    pdl_launch_dependents();
    const int t0 = blockIdx.x * kRtTok, e0 = blockIdx.z * kRtExp, split = blockIdx.y, tid = threadIdx.x;
    const int kq = d / nsplit, kbeg = split * kq, nch = kq / kRtK;
    // experts 8eg..8eg+7, tokens 4tg..4tg+3; tokens vary along a half-warp, so a warp's reads of
    // the expert rows are broadcasts and its reads of the token rows are 256 contiguous bytes
    const int tg = tid & 15, eg = tid >> 4;
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    // global -> register staging: W rows (e fastest across threads) and x rows
    float4 wr[4], xr[2];
    const float rc = router_input_scale(d);
    float ns[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int t = (tid + 256 * i) & 63;
        ns[i] = nscale && t0 + t < T ? nscale[t0 + t] : 1.f;
    }
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = tid + 256 * i, e = idx & 127, qd = idx >> 7;
            wr[i] = e0 + e < E ? __ldg(reinterpret_cast<const float4 *>(W + (size_t)(e0 + e) * d + k0 + 4 * qd))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + 256 * i, t = idx & 63, qd = idx >> 6;
            xr[i] = t0 + t < T ? __ldg(reinterpret_cast<const float4 *>(x + (size_t)(t0 + t) * d + k0 + 4 * qd))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            if (nscale) xr[i] = router_input4(xr[i], ns[i], rc, __ldg(reinterpret_cast<const float4 *>(rscale + k0 + 4 * qd)));
        }
    };
    auto store = [&]() {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = tid + 256 * i, e = idx & 127, qd = idx >> 7;
            ws[4 * qd][e] = wr[i].x; ws[4 * qd + 1][e] = wr[i].y; ws[4 * qd + 2][e] = wr[i].z; ws[4 * qd + 3][e] = wr[i].w;
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + 256 * i, t = idx & 63, qd = idx >> 6;
            xs[4 * qd][t] = xr[i].x; xs[4 * qd + 1][t] = xr[i].y; xs[4 * qd + 2][t] = xr[i].z; xs[4 * qd + 3][t] = xr[i].w;
        }
    };
    load(kbeg);
    for (int c = 0; c < nch; ++c) {
        store();
        __syncthreads();
        if (c + 1 < nch) load(kbeg + (c + 1) * kRtK);
#pragma unroll 8
        for (int kk = 0; kk < kRtK; ++kk) {
            const float4 wa = *reinterpret_cast<const float4 *>(&ws[kk][8 * eg]);
            const float4 wb = *reinterpret_cast<const float4 *>(&ws[kk][8 * eg + 4]);
            const float4 xv = *reinterpret_cast<const float4 *>(&xs[kk][4 * tg]);
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
            const float xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wv[i], xx[j], acc[i][j]);
        }
        __syncthreads();
    }
    float *pp = part + (size_t)split * T * E;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int t = t0 + 4 * tg + j;
        if (t >= T) continue;
        const int e = e0 + 8 * eg;   // E is a multiple of 32: the 8 experts are all present or all absent
        if (e < E) {
            float4 *dst = reinterpret_cast<float4 *>(pp + (size_t)t * E + e);
            dst[0] = make_float4(acc[0][j], acc[1][j], acc[2][j], acc[3][j]);
            dst[1] = make_float4(acc[4][j], acc[5][j], acc[6][j], acc[7][j]);
        }
    }
}

// softmax -> top-k -> normalised weights, one warp per token (same arithmetic as route_tokens)
__global__ void __launch_bounds__(256) pf_topk_kernel(const float *part, const float *bias, float *logits, int32_t *ids,
                                                      float *wts, int T, int E, int k, int nsplit) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const int per = E / 32;
    float v[kMaxE / 32];
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
        v[i] = -INFINITY;
        if (i < per) {
            // the router's K parts added in order, then the bias (ggml_add after the mul_mat)
            const size_t o = (size_t)t * E + lane + 32 * i;
            float l = part[o];
#pragma unroll
            for (int sp = 1; sp < nsplit; ++sp) l = __fadd_rn(l, part[(size_t)sp * T * E + o]);
            if (bias) l = __fadd_rn(l, bias[lane + 32 * i]);
            logits[o] = l;
            v[i] = l;
        }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) mx = fmaxf(mx, v[i]);
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) if (i < per) s += expf(v[i] - mx);
    s = warp_sum(s);
    const float inv = 1.f / s;
    uint32_t taken = 0;
    float psum = 0.f, mine = 0.f;
    int myid = 0;
    for (int j = 0; j < k; ++j) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) {
            const int e = lane + 32 * i;
            if (i < per && !((taken >> i) & 1u) && better(v[i], e, bv, bi)) { bv = v[i]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        const float pj = __fmul_rn(expf(bv - mx), inv);
        psum = __fadd_rn(psum, pj);
        if (lane == j) { myid = bi; mine = pj; }
    }
    psum = fmaxf(psum, 6.103515625e-5f);
    if (lane < k) {
        ids[(size_t)t * k + lane] = myid;
        wts[(size_t)t * k + lane] = __fdiv_rn(mine, psum);
    }
}

struct PfDispatchParams {
    const int32_t *ids;
    int32_t T, E, k;
    Residency res;
    int32_t hot_n, cold_n;     // pool sizes (0 = class absent)
    int32_t *cnt, *off, *perm, *pos;
    PfTile *tiles;
    int32_t *n_tiles;
};

// One CTA of 1024 threads. Warp w owns the contiguous pair range [w*per, (w+1)*per); counting
// and placement walk it 32 pairs at a time in pair order, so the permutation is stable.
// Lanes of the warp holding the same value as this lane (0 <= e < 256 for every lane that counts):
// the AND over the value's 8 bits of that bit's ballot or its complement. Equivalent to
// __match_any_sync, which runs far slower on this part (it dominated the dispatch kernel's time).
__device__ __forceinline__ unsigned same_lanes(int e) {
    unsigned m = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const bool on = (e >> b) & 1;
        const unsigned bb = __ballot_sync(0xffffffffu, on);
        m &= on ? bb : ~bb;
    }
    return m;
}

__global__ void __launch_bounds__(1024, 1) pf_dispatch_kernel(PfDispatchParams p) {
    __shared__ int32_t wcnt[32][kMaxE];
    __shared__ int32_t cnt[kMaxE], off[kMaxE + 1], tpre[kMaxE + 1], cls[kMaxE], widx[kMaxE];
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int P = p.T * p.k, E = p.E;
    for (int i = tid; i < 32 * kMaxE; i += 1024) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    const int per = (P + 31) / 32;
    const int lo = min(P, warp * per), hi = min(P, lo + per);
    const unsigned lt = (1u << lane) - 1u;
    // eight 32-pair steps per batch: the ids are loaded before any is counted (latency), then the
    // steps run in pair order
    for (int base = lo; base < hi; base += 256) {
        int ev[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ev[j] = base + 32 * j + lane < hi ? p.ids[base + 32 * j + lane] : -1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int e = ev[j];
            if (e >= E) { atomicOr(&g_error, ERR_BAD_EXPERT); e = 0; }
            const bool v = e >= 0;        // a negative id is an absent pair (expert-parallel partial routing)
            const unsigned act = __ballot_sync(0xffffffffu, v);
            if (act == 0u) continue;      // a step of absent pairs only (warp-uniform)
            const unsigned peers = same_lanes(e) & act;
            if (v && (peers & lt) == 0) wcnt[warp][e] += __popc(peers);
            __syncwarp();
        }
    }
    __syncthreads();
    if (tid < E) {
        int c = 0;
        for (int w = 0; w < 32; ++w) c += wcnt[w][tid];
        cnt[tid] = c;
        int cl = -1, wi = tid;
        if (c > 0) {
            if (p.res.n_slots > 0 && p.res.exp_slot) {
                const int s = p.res.exp_slot[tid];
                if (s >= 0 && s < p.res.n_slots && p.res.slot_state[s] == 2 && p.res.slot_exp[s] == tid) { cl = 0; wi = s; }
            }
            if (cl < 0 && tid < p.cold_n) cl = 1;
            if (cl == 0 && wi >= p.hot_n) cl = -1;
            if (cl < 0) atomicOr(&g_error, ERR_BAD_EXPERT);
        }
        cls[tid] = cl;
        widx[tid] = wi;
    }
    __syncthreads();
    if (warp == 0) {
        int base = 0, tb = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < E ? cnt[e] : 0;
            const int nt = (e < E && cls[e] >= 0) ? (c + kPfN - 1) / kPfN : 0;
            int ic = c, it = nt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, it, o);
                if (lane >= o) { ic += a; it += b; }
            }
            if (e < E) { off[e] = base + ic - c; tpre[e] = tb + it - nt; }
            base += __shfl_sync(0xffffffffu, ic, 31);
            tb += __shfl_sync(0xffffffffu, it, 31);
        }
        if (lane == 0) { off[E] = base; tpre[E] = tb; }
    }
    __syncthreads();
    if (tid < E) {
        int run = off[tid];
        for (int w = 0; w < 32; ++w) { const int c = wcnt[w][tid]; wcnt[w][tid] = run; run += c; }
        const int c = cnt[tid], nt = tpre[tid + 1] - tpre[tid];
        if (nt > 0) {
            const int bsz = c / nt, rem = c - bsz * nt;
            int s0 = off[tid];
            for (int i = 0; i < nt; ++i) {
                const int n = bsz + (i < rem ? 1 : 0);
                PfTile tl;
                tl.cls = cls[tid]; tl.widx = widx[tid]; tl.slot0 = s0; tl.n = n;
                p.tiles[tpre[tid] + i] = tl;
                s0 += n;
            }
        }
        if (p.cnt) p.cnt[tid] = c;
        if (p.off) p.off[tid] = off[tid];
    }
    if (tid == 0) {
        *p.n_tiles = tpre[E];
        if (p.off) p.off[E] = off[E];
    }
    __syncthreads();
    for (int base = lo; base < hi; base += 256) {
        int ev[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ev[j] = base + 32 * j + lane < hi ? p.ids[base + 32 * j + lane] : -1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int pi = base + 32 * j + lane;
            int e = ev[j];
            if (e >= E) e = 0;
            const bool v = e >= 0;
            const unsigned act = __ballot_sync(0xffffffffu, v);
            if (act == 0u) {              // a step of absent pairs only (warp-uniform)
                if (pi < hi) p.pos[pi] = -1;
                continue;
            }
            const unsigned peers = same_lanes(e) & act;
            const int b0 = v ? wcnt[warp][e] : 0;
            __syncwarp();
            if (v) {
                const int at = b0 + __popc(peers & lt);
                p.perm[at] = pi;
                p.pos[pi] = cls[e] >= 0 ? at : -1;
                if ((peers & lt) == 0) wcnt[warp][e] = b0 + __popc(peers);
            } else if (pi < hi) {
                p.pos[pi] = -1;
            }
            __syncwarp();
        }
    }
}

// Q8_K quantisation of every token: one warp per (token, super-block)
__global__ void __launch_bounds__(256) pf_actq_kernel(const float *x, int8_t *xq8, float *xd, int16_t *xbs, int T,
                                                      int d) {
    pdl_wait();
    pdl_launch_dependents();
    const int nsb = d / QK_K;
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (item >= T * nsb) return;
    const int t = item / nsb, sb = item - t * nsb;
    q8k_superblock_warp(x + (size_t)t * d + sb * QK_K, xq8 + (size_t)t * d + sb * QK_K, xd + item, xbs + (size_t)item * 16,
                        lane);
}

// Q8_K rows already quantised by the sender (the expert-parallel exchange carries them instead of
// f32 rows), ggml layout per super-block: d f32 | qs[256] | bsums[16] i16 (292 bytes), split into the
// xq8 / xd / xbs arrays pf_actq_kernel writes. One warp per (token, super-block), 73 words.
__global__ void __launch_bounds__(256) pf_unpack_q8k_kernel(const uint8_t *rows, int8_t *xq8, float *xd, int16_t *xbs,
                                                            int T, int d) {
    pdl_wait();
    pdl_launch_dependents();
    const int nsb = d / QK_K;
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (item >= T * nsb) return;
    const int t = item / nsb, sb = item - t * nsb;
    const uint32_t *src = reinterpret_cast<const uint32_t *>(rows + (size_t)item * B_Q8_K);
    uint32_t *qs = reinterpret_cast<uint32_t *>(xq8 + (size_t)t * d + sb * QK_K);
    uint32_t *bs = reinterpret_cast<uint32_t *>(xbs + (size_t)item * 16);
    for (int i = lane; i < B_Q8_K / 4; i += 32) {
        const uint32_t v = __ldg(src + i);
        if (i == 0) xd[item] = __uint_as_float(v);
        else if (i <= QK_K / 4) qs[i - 1] = v;
        else bs[i - 1 - QK_K / 4] = v;
    }
}

// The Gemma-4 block norms' first kernel (in place of pf_actq_kernel, ahead of the router): per
// token its rms_norm scale (written for the router) and the Q8_K rows of the expert input
// rms_norm(x) * pre. One CTA per token, one warp per 256-value super-block: the squares of the
// warp's values summed in double, the warps' sums added in warp order.
__global__ void __launch_bounds__(kPrefillMaxSb * 32) pf_actq_norm_kernel(const float *x, int8_t *xq8, float *xd,
                                                                         int16_t *xbs, float *nscale, const float *pre,
                                                                         int T, int d, float eps) {
    __shared__ double red[kPrefillMaxSb];
    __shared__ float sc;
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x, sb = threadIdx.x >> 5, lane = threadIdx.x & 31, nsb = d / QK_K;
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)t * d + sb * QK_K);
    const float4 a = __ldg(x4 + 2 * lane), b = __ldg(x4 + 2 * lane + 1);
    const double sq = warp_sum_d(sq_sum4(a) + sq_sum4(b));
    if (lane == 0) red[sb] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int i = 0; i < nsb; ++i) tot += red[i];
        sc = rms_row_scale(tot, d, eps);
        nscale[t] = sc;
    }
    __syncthreads();
    const float s = sc;
    const float4 *w4 = reinterpret_cast<const float4 *>(pre + sb * QK_K);
    const float4 na = norm_weight4(a, s, __ldg(w4 + 2 * lane)), nb = norm_weight4(b, s, __ldg(w4 + 2 * lane + 1));
    float v[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
    const int item = t * nsb + sb;
    q8k_quantize_warp(v, xq8 + (size_t)t * d + sb * QK_K, xd + item, xbs + (size_t)item * 16, lane);
}

// out[t] = ((w0 y0 + w1 y1) + w2 y2) + ...: products rounded, then added in slot order, as the
// reference's mul + add chain does; optionally copies y to pair order. With post given (the
// Gemma-4 ffn_post_norm_2) the row is then rms-normed and multiplied by post.
constexpr int kCbThreads = 256, kCbPer = kPrefillMaxSb * QK_K / (4 * kCbThreads);
__global__ void __launch_bounds__(kCbThreads) pf_combine_kernel(const float *y, const int32_t *pos, const float *w,
                                                                float *out, float *y_pairs, int T, int k, int d,
                                                                const float *post, float eps) {
    __shared__ double red[kCbThreads / 32];
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    float4 row[kCbPer];
    double sq = 0.0;
#pragma unroll
    for (int it = 0; it < kCbPer; ++it) {
        const int c = 4 * (threadIdx.x + it * kCbThreads);
        if (c >= d) break;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; ++j) {
            const int sl = pos[(size_t)t * k + j];
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (sl >= 0) v = *reinterpret_cast<const float4 *>(y + (size_t)sl * d + c);
            const float wj = w[(size_t)t * k + j];
            const float4 pr = make_float4(__fmul_rn(wj, v.x), __fmul_rn(wj, v.y), __fmul_rn(wj, v.z), __fmul_rn(wj, v.w));
            if (j == 0) acc = pr;
            else acc = make_float4(__fadd_rn(acc.x, pr.x), __fadd_rn(acc.y, pr.y), __fadd_rn(acc.z, pr.z), __fadd_rn(acc.w, pr.w));
            if (y_pairs) *reinterpret_cast<float4 *>(y_pairs + ((size_t)t * k + j) * d + c) = v;
        }
        row[it] = acc;
        sq += sq_sum4(acc);
        if (!post) *reinterpret_cast<float4 *>(out + (size_t)t * d + c) = acc;
    }
    if (!post) return;
    sq = warp_sum_d(sq);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    double tot = 0.0;   // the warps' sums in warp order
#pragma unroll
    for (int i = 0; i < kCbThreads / 32; ++i) tot += red[i];
    const float sc = rms_row_scale(tot, d, eps);
#pragma unroll
    for (int it = 0; it < kCbPer; ++it) {
        const int c = 4 * (threadIdx.x + it * kCbThreads);
        if (c >= d) break;
        *reinterpret_cast<float4 *>(out + (size_t)t * d + c) =
            norm_weight4(row[it], sc, __ldg(reinterpret_cast<const float4 *>(post + c)));
    }
}

}  // namespace moeb
