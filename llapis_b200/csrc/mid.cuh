// Mid-size batches (tens of routed pairs per expert): grouped GEMMs on warp-level int8 MMAs over the
// weights' own integer codes, so no weight element is ever converted to a float operand.
//
// Same routing, dispatch, Q8_K activation and combine kernels as the prefill path (prefill.cuh);
// between them:
//   md_bimg_kernel      Q8_K activations -> gate_up operand image (fragment order, per 8-pair column
//                       block of each dispatch tile)
//   md_kernel<0>        gate_up: Q4_K / IQ2_S rows x image -> h[slot][2 n_ff] (f32)
//   md_act_kernel       GeGLU (fp16-table GELU) + Q8_0 of h -> down operand image
//   md_kernel<1>        down: Q5_0 / IQ4_NL rows x image -> y[slot][d] (x per-expert scale)
//
// md_kernel is a persistent kernel (one CTA per SM): a producer warp streams 16-row stages of the
// tiles' weight rows from HBM into a ring of shared-memory slots with bulk copies; 16 consumer warps in
// 4 groups claim the stages in order. The 4 warps of a group split the stage's K range (super-blocks
// wg, wg + 4, ... of the row), loop over the tile's 8-pair column blocks with m16n8k32 / m16n8k16 s8
// MMAs, and add their four partial tiles in a fixed order through shared memory. The integer work per
// 32 (or 16) K elements is exact, as in the reference's vec_dot kernels (ggml-cpu/arch/x86/quants.c:
// ggml_vec_dot_q4_K_q8_K, _iq2_s_q8_K, _q5_0_q8_0, _iq4_nl_q8_0); the float scaling and the order of
// the float additions differ from the reference, within the output tolerance.

#pragma once

namespace moeb {

constexpr int kMdWarps = 16;                  // consumer warps
constexpr int kMdGroups = 4;
constexpr int kMdThreads = (kMdWarps + 1) * 32;
constexpr int kMdRows = 16;                   // weight rows per stage (one MMA M tile)
constexpr int kMdMaxTiles = 512;
constexpr int kMdMaxUnits = 1024;
constexpr int kMdMaxSlots = 16;
constexpr int kMdTileStride = 48;             // bytes per row of a decoded 16 x 32 A tile (conflict-free ldmatrix)
// operand images, per 8-pair column block: gate_up per super-block 4 x 512 B of q8 words (lane order)
// then 512 B of {min-term word, dx of columns 2c and 2c + 1}; down per 32-block 512 B of {q8 words of
// K 4c.. and 16 + 4c.., dx of columns 2c and 2c + 1}
constexpr int kMdGuSbBytes = 5 * 512;
constexpr int kMdDnBlkBytes = 512;
static_assert(kMdMaxTiles <= kMdWarps * 32 && kMdMaxUnits <= 2 * kMdWarps * 32, "one scan pass");

// column blocks per work unit: a unit's operand chunk stays in shared memory for all its stages
template <int KIND> struct MdCfg { static constexpr int kChunk = KIND == 0 ? 2 : 4; };
__host__ __device__ inline int md_chunk(int kind) { return kind == 0 ? 2 : 4; }

__host__ __device__ inline size_t md_cb_bytes(int kind, int d, int nff) {
    return kind == 0 ? (size_t)(d / QK_K) * kMdGuSbBytes : (size_t)(nff / QK32) * kMdDnBlkBytes;
}

struct MdParams {
    int32_t T, E, d, k, nff;
    PoolView pv[2];                // this kind's hot / cold pools
    const PfTile *tiles;
    const int32_t *n_tiles;
    const int32_t *perm;
    const uint8_t *img;            // operand image of this kind
    float *out;                    // h (gate_up) or y (down), slot order
};

// Work units: (dispatch tile, chunk of kChunk column blocks); every unit covers all the tile's weight
// rows, so the CTA split runs over (unit, 8-row group) positions weighted by each unit's cost.
struct MdShared {
    int32_t n_tiles, n_units;
    int32_t cls[kMdMaxTiles], widx[kMdMaxTiles], slot0[kMdMaxTiles], n[kMdMaxTiles], cb0[kMdMaxTiles];
    int32_t ufirst[kMdMaxTiles];       // first unit of each tile
    int16_t utile[kMdMaxUnits];
    uint32_t pre[kMdMaxUnits + 1];     // cumulative work units
    int32_t scan_a[kMdWarps + 1];
    uint32_t scan_b[kMdWarps + 1];
    int32_t split[2];
    int32_t claim_cnt[2];              // stages claimed of the current unit (by unit parity)
    int32_t claim[kMdGroups][2];
};

// smem layout of md_kernel: the ring gets every byte left under 227 KB (up to kMdMaxSlots slots)
struct MdLayout {
    int sh, bars, grid, part, atile, bchunk, slots, slot_cap, n_slots, total;
};
__host__ __device__ inline MdLayout md_layout(int kind, int d, int nff) {
    MdLayout L;
    const int ch = md_chunk(kind);
    int o = 0;
    L.sh = o;     o += (int)((sizeof(MdShared) + 127) / 128 * 128);
    L.bars = o;   o += ((2 * kMdMaxSlots + 1) * 8 + 127) / 128 * 128;
    L.grid = o;   o += kind == 0 ? MOE_IQ2S_GRID_ROWS * 8 : 0;
    L.part = o;   o += kMdWarps * kMdRows * (8 * ch + 1) * 4;          // a 16 x 8ch f32 partial tile per warp
    o = (o + 15) / 16 * 16;
    L.atile = o;  o += kMdWarps * 2 * kMdRows * kMdTileStride;          // two decoded A tiles per warp
    o = (o + 127) / 128 * 128;
    L.bchunk = o; o += (int)(ch * md_cb_bytes(kind, d, nff));
    o = (o + 127) / 128 * 128;
    L.slots = o;
    const int rb = kind == 0 ? (int)row_bytes(T_Q4_K, d) : (int)row_bytes(T_Q5_0, nff);
    L.slot_cap = (kMdRows * rb + 16 + 127) / 128 * 128;
    L.n_slots = (227 * 1024 - o) / L.slot_cap;
    if (L.n_slots > kMdMaxSlots) L.n_slots = kMdMaxSlots;
    o += (L.n_slots > 0 ? L.n_slots : 0) * L.slot_cap;
    L.total = o;
    return L;
}

// Tiles and work units into shared memory. Thread t owns tile t: its column blocks and units; unit
// costs per 8-row group weigh the bytes streamed (x 3 instructions per byte at the measured
// bandwidth) against the consumer instructions, which grow with the unit's column blocks. The bases
// are scans (warp shuffles, then the preceding warps' totals).
template <int KIND>
__device__ void md_load_tiles(const MdParams &p, MdShared &sh, int tid) {
    constexpr int CH = MdCfg<KIND>::kChunk;
    const int lane = tid & 31, warp = tid >> 5;
    const int nt = min(*p.n_tiles, kMdMaxTiles);
    if (tid == 0 && *p.n_tiles > kMdMaxTiles) atomicOr(&g_error, ERR_CAPACITY);
    const int d_in = KIND == 0 ? p.d : p.nff;
    const int gpe = (KIND == 0 ? 2 * p.nff : p.d) / kGroupRows;
    int ncb = 0, nch = 0;
    if (tid < nt) {
        const PfTile tl = p.tiles[tid];
        sh.cls[tid] = tl.cls; sh.widx[tid] = tl.widx; sh.slot0[tid] = tl.slot0; sh.n[tid] = tl.n;
        ncb = (tl.n + 7) / 8;
        nch = (ncb + CH - 1) / CH;
    }
    int ci = ncb, ui = nch;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, ci, o), b = __shfl_up_sync(0xffffffffu, ui, o);
        if (lane >= o) { ci += a; ui += b; }
    }
    if (lane == 31) { sh.scan_a[warp] = ci; sh.scan_b[warp] = (uint32_t)ui; }
    __syncthreads();
    for (int w = 0; w < warp; ++w) { ci += sh.scan_a[w]; ui += (int)sh.scan_b[w]; }
    if (tid < nt) {
        sh.cb0[tid] = ci - ncb;
        const int u0 = ui - nch;
        sh.ufirst[tid] = u0;
        for (int c = 0; c < nch && u0 + c < kMdMaxUnits; ++c) sh.utile[u0 + c] = (int16_t)tid;
        if (tid == nt - 1) sh.n_units = min(ui, kMdMaxUnits);
        if (tid == nt - 1 && ui > kMdMaxUnits) atomicOr(&g_error, ERR_CAPACITY);
    }
    if (tid == 0 && nt == 0) sh.n_units = 0;
    __syncthreads();
    // unit costs, two units per thread, then the scan
    const int nu = sh.n_units;
    uint32_t c2[2] = {0u, 0u};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int u = 2 * tid + h;
        if (u < nu) {
            const int t = sh.utile[u], ch = u - sh.ufirst[t];
            const int ncb_t = (sh.n[t] + 7) / 8, nc = min(CH, ncb_t - ch * CH);
            const int type = p.pv[sh.cls[t] == 0 ? 0 : 1].type;
            const uint32_t bytes = 8u * (uint32_t)row_bytes(type, d_in);
            const uint32_t kunits = KIND == 0 ? (uint32_t)(d_in / QK_K) * 8u : (uint32_t)(d_in / QK32);
            const uint32_t dec = KIND == 0 ? (type == T_IQ2_S ? 60u : 12u) : (type == T_IQ4_NL ? 30u : 36u);
            c2[h] = (3u * bytes + 16u * kunits * (dec + 14u * (uint32_t)nc)) / 64u * (uint32_t)gpe;
        }
    }
    uint32_t gi = c2[0] + c2[1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t b = __shfl_up_sync(0xffffffffu, gi, o);
        if (lane >= o) gi += b;
    }
    __syncthreads();   // scan_b reused
    if (lane == 31) sh.scan_b[warp] = gi;
    __syncthreads();
    for (int w = 0; w < warp; ++w) gi += sh.scan_b[w];
    if (2 * tid < nu) sh.pre[2 * tid + 1] = gi - c2[1];
    if (2 * tid + 1 < nu) sh.pre[2 * tid + 2] = gi;
    if (tid == 0) {
        sh.pre[0] = 0;
        sh.n_tiles = nt;
    }
    __syncthreads();
}

// ---- per-format consumers: one warp, its K part, column blocks [0, nc) of the unit's operand chunk
// in shared memory (blocks cbb bytes apart); out[q][i]: rows g / g + 8, columns 2c / 2c + 1

// Q4_K rows (gate_up): ggml_vec_dot_q4_K_q8_K's integer work on MMAs straight from the stage's
// nibbles; per sub-block j an m16n8k32 gives sum_i q_i * q8_i, scaled by the 6-bit sc_j in int32; the
// min term sum_j m_j * bsum_j runs as two m16n8k16 (bsum = 64 hi + lo).
template <int CH>
__device__ __forceinline__ void md_q4k(const uint8_t *stage, uint32_t stage_s, int rb, int nsb, int wg,
                                       const uint8_t *img, size_t cbb, int nc, float (&out)[CH][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3, am = lane >> 3;
    const uint32_t a_row = stage_s + (uint32_t)(((lane & 7) + 8 * (am & 1)) * rb + 16 * (am >> 1) + 16);
    const uint8_t *r0 = stage + (size_t)g * rb, *r1 = stage + (size_t)(g + 8) * rb;
    const uint32_t M = 0x0f0f0f0fu;
#pragma unroll 1
    for (int sb = wg; sb < nsb; sb += 4) {
        const uint4 h0 = *reinterpret_cast<const uint4 *>(r0 + sb * B_Q4_K);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(r1 + sb * B_Q4_K);
        // 6-bit scales / mins of sub-blocks 0-3 and 4-7, four per word (get_scale_min_k4, ggml-quants.c:822)
        const uint32_t s0l = h0.y & 0x3f3f3f3fu, s0h = (h0.w & M) | ((h0.y >> 2) & 0x30303030u);
        const uint32_t m0l = h0.z & 0x3f3f3f3fu, m0h = ((h0.w >> 4) & M) | ((h0.z >> 2) & 0x30303030u);
        const uint32_t s1l = h1.y & 0x3f3f3f3fu, s1h = (h1.w & M) | ((h1.y >> 2) & 0x30303030u);
        const uint32_t m1l = h1.z & 0x3f3f3f3fu, m1h = ((h1.w >> 4) & M) | ((h1.z >> 2) & 0x30303030u);
        const uint8_t *isb = img + (size_t)sb * kMdGuSbBytes + lane * 16;
        int as[CH][4];
#pragma unroll
        for (int q = 0; q < CH; ++q) as[q][0] = as[q][1] = as[q][2] = as[q][3] = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t w0, w1, w2, w3;
            ldsm_x4(a_row + (uint32_t)(sb * B_Q4_K + 32 * i), w0, w1, w2, w3);
            const uint32_t l0 = w0 & M, l1 = w1 & M, l2 = w2 & M, l3 = w3 & M;
            const uint32_t u0 = (w0 >> 4) & M, u1 = (w1 >> 4) & M, u2 = (w2 >> 4) & M, u3 = (w3 >> 4) & M;
            const int jl = 2 * i, jh = 2 * i + 1;
            const int sl0 = sbyte(jl < 4 ? s0l : s0h, jl & 3), sh0 = sbyte(jh < 4 ? s0l : s0h, jh & 3);
            const int sl1 = sbyte(jl < 4 ? s1l : s1h, jl & 3), sh1 = sbyte(jh < 4 ? s1l : s1h, jh & 3);
#pragma unroll
            for (int q = 0; q < CH; ++q) {
                if (q < nc) {
                    const uint4 b = *(reinterpret_cast<const uint4 *>(isb + (size_t)q * cbb + i * 512));
                    int dl[4], dh[4];
                    mma_s8_k32(dl, l0, l1, l2, l3, b.x, b.y);
                    mma_s8_k32(dh, u0, u1, u2, u3, b.z, b.w);
                    as[q][0] += sl0 * dl[0] + sh0 * dh[0];
                    as[q][1] += sl0 * dl[1] + sh0 * dh[1];
                    as[q][2] += sl1 * dl[2] + sh1 * dh[2];
                    as[q][3] += sl1 * dl[3] + sh1 * dh[3];
                }
            }
        }
        const uint32_t am0 = (c & 1) ? m0h : m0l, am1 = (c & 1) ? m1h : m1l;
        const float dw0 = h2f((uint16_t)(h0.x & 0xffffu)), dm0 = h2f((uint16_t)(h0.x >> 16));
        const float dw1 = h2f((uint16_t)(h1.x & 0xffffu)), dm1 = h2f((uint16_t)(h1.x >> 16));
#pragma unroll
        for (int q = 0; q < CH; ++q) {
            if (q < nc) {
                const uint4 mb = *(reinterpret_cast<const uint4 *>(isb + (size_t)q * cbb + 2048));
                int d1[4], d2[4];
                mma_s8_k16(d1, am0, am1, c < 2 ? mb.x : 0u);
                mma_s8_k16(d2, am0, am1, c < 2 ? 0u : mb.x);
                const float dxa = __uint_as_float(mb.y), dxb = __uint_as_float(mb.z);
                out[q][0] = fmaf(dxa, fmaf(-dm0, (float)(64 * d1[0] + d2[0]), dw0 * (float)as[q][0]), out[q][0]);
                out[q][1] = fmaf(dxb, fmaf(-dm0, (float)(64 * d1[1] + d2[1]), dw0 * (float)as[q][1]), out[q][1]);
                out[q][2] = fmaf(dxa, fmaf(-dm1, (float)(64 * d1[2] + d2[2]), dw1 * (float)as[q][2]), out[q][2]);
                out[q][3] = fmaf(dxb, fmaf(-dm1, (float)(64 * d1[3] + d2[3]), dw1 * (float)as[q][3]), out[q][3]);
            }
        }
    }
}

// IQ2_S rows (gate_up): each lane decodes 16 values (two 8-value grid entries with their signs) of
// the 16 x 32 tile of a sub-block into shared memory, the warp reads the MMA fragments back with
// ldmatrix, and every 16-value half runs as one m16n8k16 with its own scale 2 s + 1 (int32). Times
// d_w * d_x per super-block; the caller multiplies by 0.125 (ggml_vec_dot_iq2_s_q8_K).
template <int CH>
__device__ __forceinline__ void md_iq2s(const uint8_t *stage, int rb, int nsb, int wg, const uint64_t *grid,
                                        uint8_t *atile, const uint8_t *img, size_t cbb, int nc,
                                        float (&out)[CH][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, am = lane >> 3;
    const int dr = lane >> 1, dh = lane & 1;   // decode: row, 16-value half
    const uint8_t *rd = stage + (size_t)dr * rb;
    const uint8_t *r0 = stage + (size_t)g * rb, *r1 = stage + (size_t)(g + 8) * rb;
    const uint32_t at_s = smem_addr(atile);
    const uint32_t a_off = (uint32_t)(((lane & 7) + 8 * (am & 1)) * kMdTileStride + 16 * (am >> 1));
    int buf = 0;
#pragma unroll 1
    for (int sb = wg; sb < nsb; sb += 4) {
        const uint8_t *bd = rd + sb * B_IQ2_S;
        const float dw0 = h2f(*reinterpret_cast<const uint16_t *>(r0 + sb * B_IQ2_S));
        const float dw1 = h2f(*reinterpret_cast<const uint16_t *>(r1 + sb * B_IQ2_S));
        const uint8_t *isb = img + (size_t)sb * kMdGuSbBytes + lane * 16;
        int is[CH][4];
#pragma unroll
        for (int q = 0; q < CH; ++q) is[q][0] = is[q][1] = is[q][2] = is[q][3] = 0;
#pragma unroll 2
        for (int j = 0; j < 8; ++j) {
            // decode: grid entries l = 2 dh, 2 dh + 1 of sub-block j of row dr
            const uint32_t q2 = *reinterpret_cast<const uint16_t *>(bd + 2 + 4 * j + 2 * dh);
            const uint32_t s2 = *reinterpret_cast<const uint16_t *>(bd + 34 + 4 * j + 2 * dh);
            const uint32_t qh = bd[66 + j];
            uint32_t v[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int l = 2 * dh + h;
                const uint32_t gi = ((q2 >> (8 * h)) & 0xffu) | (((qh >> (2 * l)) & 3u) << 8);
                const uint64_t gv = grid[gi];
                const uint32_t s = (s2 >> (8 * h)) & 0xffu;
                const uint32_t c0 = ((s & 15u) * 0x00204081u) & 0x01010101u;
                const uint32_t c1 = ((s >> 4) * 0x00204081u) & 0x01010101u;
                // negate flagged bytes: (w ^ 0xff) + 1 == -w; magnitudes are >= 8, so nothing carries
                v[2 * h] = ((uint32_t)gv ^ (c0 * 0xffu)) + c0;
                v[2 * h + 1] = ((uint32_t)(gv >> 32) ^ (c1 * 0xffu)) + c1;
            }
            uint8_t *tw = atile + buf * (kMdRows * kMdTileStride);
            *reinterpret_cast<uint4 *>(tw + dr * kMdTileStride + 16 * dh) = make_uint4(v[0], v[1], v[2], v[3]);
            __syncwarp();
            uint32_t a0, a1, a2, a3;
            ldsm_x4(at_s + (uint32_t)(buf * (kMdRows * kMdTileStride)) + a_off, a0, a1, a2, a3);
            buf ^= 1;
            const uint32_t sc0 = r0[sb * B_IQ2_S + 74 + j], sc1 = r1[sb * B_IQ2_S + 74 + j];
            const int ls00 = 1 + 2 * (int)(sc0 & 15u), ls01 = 1 + 2 * (int)(sc0 >> 4);
            const int ls10 = 1 + 2 * (int)(sc1 & 15u), ls11 = 1 + 2 * (int)(sc1 >> 4);
#pragma unroll
            for (int q = 0; q < CH; ++q) {
                if (q < nc) {
                    const uint4 b = *(reinterpret_cast<const uint4 *>(isb + (size_t)q * cbb + (j >> 1) * 512));
                    const uint32_t blo = (j & 1) ? b.z : b.x, bhi = (j & 1) ? b.w : b.y;
                    int d0[4], d1[4];
                    mma_s8_k16(d0, a0, a1, blo);
                    mma_s8_k16(d1, a2, a3, bhi);
                    is[q][0] += ls00 * d0[0] + ls01 * d1[0];
                    is[q][1] += ls00 * d0[1] + ls01 * d1[1];
                    is[q][2] += ls10 * d0[2] + ls11 * d1[2];
                    is[q][3] += ls10 * d0[3] + ls11 * d1[3];
                }
            }
        }
#pragma unroll
        for (int q = 0; q < CH; ++q) {
            if (q < nc) {
                const uint4 mb = *(reinterpret_cast<const uint4 *>(isb + (size_t)q * cbb + 2048));
                const float dxa = __uint_as_float(mb.y), dxb = __uint_as_float(mb.z);
                out[q][0] = fmaf(dw0 * dxa, (float)is[q][0], out[q][0]);
                out[q][1] = fmaf(dw0 * dxb, (float)is[q][1], out[q][1]);
                out[q][2] = fmaf(dw1 * dxa, (float)is[q][2], out[q][2]);
                out[q][3] = fmaf(dw1 * dxb, (float)is[q][3], out[q][3]);
            }
        }
    }
}

// 4 bits of x -> bit 4 of each byte
__device__ __forceinline__ uint32_t md_spread4(uint32_t x) { return ((x & 15u) * 0x02040810u) & 0x10101010u; }

// Q5_0 / IQ4_NL rows (down): each lane decodes 16 values of the 16 x 32 tile of a 32-block (qs
// bytes 8 h .. 8 h + 7, both nibbles) into shared memory as signed int8; one m16n8k32 per block
// and column block, times d_w * d_x in f32 (ggml_vec_dot_q5_0_q8_0 / ggml_vec_dot_iq4_nl_q8_0).
template <int CH>
__device__ __forceinline__ void md_down(const uint8_t *stage, int rb, int nb, int wg, int type,
                                        const uint32_t (&kv)[4], uint8_t *atile, const uint8_t *img, size_t cbb,
                                        int nc, float (&out)[CH][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, am = lane >> 3;
    const int dr = lane >> 1, dh = lane & 1;
    const uint8_t *rd = stage + (size_t)dr * rb;
    const uint8_t *r0 = stage + (size_t)g * rb, *r1 = stage + (size_t)(g + 8) * rb;
    const uint32_t at_s = smem_addr(atile);
    const uint32_t a_off = (uint32_t)(((lane & 7) + 8 * (am & 1)) * kMdTileStride + 16 * (am >> 1));
    const int bb = type == T_IQ4_NL ? B_IQ4_NL : B_Q5_0;
    const uint32_t M = 0x0f0f0f0fu;
    int buf = 0;
#pragma unroll 1
    for (int b = wg; b < nb; b += 4) {
        const uint8_t *blk = rd + b * bb;
        uint32_t lo0, lo1, hi0, hi1;
        if (type == T_IQ4_NL) {
            uint32_t w[2];
            lds_words_a2<2>(blk + 2 + 8 * dh, w);
            lo0 = (uint32_t)iq4nl_lookup4(w[0], kv[0], kv[1], kv[2], kv[3]);
            lo1 = (uint32_t)iq4nl_lookup4(w[1], kv[0], kv[1], kv[2], kv[3]);
            hi0 = (uint32_t)iq4nl_lookup4(w[0] >> 4, kv[0], kv[1], kv[2], kv[3]);
            hi1 = (uint32_t)iq4nl_lookup4(w[1] >> 4, kv[0], kv[1], kv[2], kv[3]);
        } else {
            uint32_t wh[1], w[2];
            lds_words_a2<1>(blk + 2, wh);            // qh
            lds_words_a2<2>(blk + 6 + 8 * dh, w);    // qs bytes 8 dh .. 8 dh + 7
            const uint32_t qh = wh[0];
            // value = (nibble | hbit << 4) - 16
            lo0 = __vsub4((w[0] & M) | md_spread4(qh >> (8 * dh)), 0x10101010u);
            lo1 = __vsub4((w[1] & M) | md_spread4(qh >> (8 * dh + 4)), 0x10101010u);
            hi0 = __vsub4(((w[0] >> 4) & M) | md_spread4(qh >> (16 + 8 * dh)), 0x10101010u);
            hi1 = __vsub4(((w[1] >> 4) & M) | md_spread4(qh >> (20 + 8 * dh)), 0x10101010u);
        }
        uint8_t *tw = atile + buf * (kMdRows * kMdTileStride) + dr * kMdTileStride;
        *reinterpret_cast<uint2 *>(tw + 8 * dh) = make_uint2(lo0, lo1);
        *reinterpret_cast<uint2 *>(tw + 16 + 8 * dh) = make_uint2(hi0, hi1);
        __syncwarp();
        uint32_t a0, a1, a2, a3;
        ldsm_x4(at_s + (uint32_t)(buf * (kMdRows * kMdTileStride)) + a_off, a0, a1, a2, a3);
        buf ^= 1;
        const float dw0 = h2f(*reinterpret_cast<const uint16_t *>(r0 + b * bb));
        const float dw1 = h2f(*reinterpret_cast<const uint16_t *>(r1 + b * bb));
        const uint8_t *ib = img + (size_t)b * kMdDnBlkBytes + lane * 16;
#pragma unroll
        for (int q = 0; q < CH; ++q) {
            if (q < nc) {
                const uint4 x = *(reinterpret_cast<const uint4 *>(ib + (size_t)q * cbb));
                int dd[4];
                mma_s8_k32(dd, a0, a1, a2, a3, x.x, x.y);
                const float dxa = __uint_as_float(x.z), dxb = __uint_as_float(x.w);
                out[q][0] = fmaf(dw0 * dxa, (float)dd[0], out[q][0]);
                out[q][1] = fmaf(dw0 * dxb, (float)dd[1], out[q][1]);
                out[q][2] = fmaf(dw1 * dxa, (float)dd[2], out[q][2]);
                out[q][3] = fmaf(dw1 * dxb, (float)dd[3], out[q][3]);
            }
        }
    }
}

#ifdef MOEB_TRACE
// per CTA (first 64), per stage of group 0: claimed, data ready, computed, reduced; per unit: start, chunk ready
__device__ unsigned long long g_mdtrace[2][64][64][4];
__device__ unsigned long long g_mdutrace[2][64][8][2];
#define MDTRACE(it, f) do { if (blockIdx.x < 64 && (it) < 64 && lane == 0 && warp == 0) g_mdtrace[KIND][blockIdx.x][it][f] = clock64(); } while (0)
#define MDUTRACE(u, f) do { if (blockIdx.x < 64 && (u) < 8 && lane == 0 && warp == 0) g_mdutrace[KIND][blockIdx.x][u][f] = clock64(); } while (0)
#else
#define MDTRACE(it, f) do { } while (0)
#define MDUTRACE(u, f) do { } while (0)
#endif

template <int KIND>
__global__ void __launch_bounds__(kMdThreads, 1) md_kernel(MdParams p) {
    constexpr int CH = MdCfg<KIND>::kChunk, PS = 8 * CH + 1;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const MdLayout L = md_layout(KIND, p.d, p.nff);
    MdShared &sh = *reinterpret_cast<MdShared *>(smem + L.sh);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + L.n_slots;
    uint64_t *bfull = empty + L.n_slots;   // the unit's operand chunk landed
    uint64_t *grid = reinterpret_cast<uint64_t *>(smem + L.grid);
    float *part = reinterpret_cast<float *>(smem + L.part);
    const uint8_t *bchunk = smem + L.bchunk;
    uint8_t *slots = smem + L.slots;
    const int d_in = KIND == 0 ? p.d : p.nff, d_out = KIND == 0 ? 2 * p.nff : p.d;
    if (tid == 0) {
        for (int s = 0; s < L.n_slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarpsPerGroup);
        }
        mbar_init(bfull, 1);
        fence_mbar_init();
        sh.claim_cnt[0] = sh.claim_cnt[1] = 0;
    }
    if (KIND == 0)
        for (int i = tid; i < MOE_IQ2S_GRID_ROWS; i += kMdThreads) grid[i] = g_iq2s_grid[i];
    pdl_wait();
    md_load_tiles<KIND>(p, sh, tid);
    pdl_launch_dependents();
    const int U = sh.n_units;
    const int gpe = d_out / kGroupRows, sg = kMdRows / kGroupRows, spe = gpe / sg;
    if (warp < 2) {
        const uint32_t pos = (uint32_t)((uint64_t)sh.pre[U] * (blockIdx.x + (uint32_t)warp) / gridDim.x);
        const int gg = group_at_pre_warp(sh.pre, U, pos, gpe, lane);
        if (lane == 0) sh.split[warp] = gg;
    }
    __syncthreads();
    const int g0 = sh.split[0], g1 = sh.split[1];
    if (g1 <= g0) return;   // no barrier below involves a CTA without work
    const int S0 = stage_of(g0, gpe, spe, sg);
    const size_t cbb = md_cb_bytes(KIND, p.d, p.nff);
    const int grp = warp / kWarpsPerGroup, wg = warp % kWarpsPerGroup, gl = tid & (kWarpsPerGroup * 32 - 1);
    uint8_t *atile = smem + L.atile + warp * 2 * kMdRows * kMdTileStride;
    float *mypart = part + warp * (kMdRows * PS);
    uint32_t kv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        kv[i] = (uint32_t)(uint8_t)g_iq4nl[4 * i] | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 1] << 8) |
                ((uint32_t)(uint8_t)g_iq4nl[4 * i + 2] << 16) | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 3] << 24);
    bool ok = true;
    const int u_lo = g0 / gpe, u_hi = (g1 - 1) / gpe;
    for (int u = u_lo; u <= u_hi; ++u) {
        // ---- unit u: its operand chunk, then its stages [su0, su1) of this CTA's stage sequence
        const int lo = max(g0, u * gpe), hi = min(g1, (u + 1) * gpe);
        const int su0 = stage_of(lo, gpe, spe, sg) - S0, su1 = stage_of(hi - 1, gpe, spe, sg) - S0 + 1;
        const int t = sh.utile[u], c0 = (u - sh.ufirst[t]) * CH, ncb = (sh.n[t] + 7) / 8, nc = min(CH, ncb - c0);
        __syncthreads();   // the previous unit is consumed: its chunk buffer and claim counter are free
        // groups may claim past the end of a unit, so each unit parity has its own counter, reset one
        // unit ahead (the next barrier orders the reset before the next unit's claims)
        if (tid == 0) sh.claim_cnt[(u - u_lo + 1) & 1] = 0;
        if (warp == kMdWarps) {
            if (lane == 0) {
                const uint32_t bytes = (uint32_t)(nc * cbb);
                mbar_expect_tx(bfull, bytes);
                bulk_g2s((void *)bchunk, p.img + (size_t)(sh.cb0[t] + c0) * cbb, bytes, bfull);
                for (int it = su0; it < su1; ++it) {
                    const int slot = it % L.n_slots;
                    if (it >= L.n_slots && !mbar_wait(&empty[slot], (uint32_t)(((it / L.n_slots) - 1) & 1))) break;
                    const StagePlan st = stage_plan(S0 + it, g0, g1, gpe, spe, sg);
                    const PoolView &pv = p.pv[sh.cls[t] == 0 ? 0 : 1];
                    const int rb = (int)row_bytes(pv.type, d_in);
                    const uint32_t sbytes = (uint32_t)(st.nrows * rb);
                    mbar_expect_tx(&full[slot], sbytes);
                    bulk_g2s(slots + slot * L.slot_cap, pool_entry(pv, sh.widx[t], d_out, d_in) + (size_t)st.row0 * rb,
                             sbytes, &full[slot]);
                }
            }
            __syncwarp();   // the whole warp reaches the next unit's CTA barrier together
            continue;
        }
        MDUTRACE(u - u_lo, 0);
        if (ok && !mbar_wait(bfull, (uint32_t)((u - u_lo) & 1))) ok = false;
        MDUTRACE(u - u_lo, 1);
        const PoolView &pv = p.pv[sh.cls[t] == 0 ? 0 : 1];
        const int rb = (int)row_bytes(pv.type, d_in), n = sh.n[t];
        const float post = (KIND == 1 && pv.scale) ? pv.scale[sh.widx[t]] : 1.f;
        for (int m = 0;; ++m) {
            if (wg == 0 && lane == 0) sh.claim[grp][m & 1] = su0 + atomicAdd(&sh.claim_cnt[(u - u_lo) & 1], 1);
            group_sync(grp);
            const int it = sh.claim[grp][m & 1];
            if (it >= su1) break;
            MDTRACE(it, 0);
            const int slot = it % L.n_slots;
            if (ok && !mbar_wait(&full[slot], (uint32_t)((it / L.n_slots) & 1))) ok = false;
            MDTRACE(it, 1);
            const StagePlan st = stage_plan(S0 + it, g0, g1, gpe, spe, sg);
            const uint8_t *stage = slots + slot * L.slot_cap;
            float acc[CH][4];
#pragma unroll
            for (int q = 0; q < CH; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
            if (ok) {
                if (KIND == 0) {
                    if (pv.type == T_Q4_K)
                        md_q4k<CH>(stage, smem_addr(stage), rb, d_in / QK_K, wg, bchunk, cbb, nc, acc);
                    else
                        md_iq2s<CH>(stage, rb, d_in / QK_K, wg, grid, atile, bchunk, cbb, nc, acc);
                } else {
                    md_down<CH>(stage, rb, d_in / QK32, wg, pv.type, kv, atile, bchunk, cbb, nc, acc);
                }
            }
            MDTRACE(it, 2);
            // this warp's partial tile: [row][col] with col = 8 q + (column within the block)
            const int g = lane >> 2, c = lane & 3;
#pragma unroll
            for (int q = 0; q < CH; ++q) {
                mypart[g * PS + 8 * q + 2 * c] = acc[q][0];
                mypart[g * PS + 8 * q + 2 * c + 1] = acc[q][1];
                mypart[(g + 8) * PS + 8 * q + 2 * c] = acc[q][2];
                mypart[(g + 8) * PS + 8 * q + 2 * c + 1] = acc[q][3];
            }
            group_sync(grp);
            // the group adds its four partial tiles in warp order and stores rows (slot order)
            const int ws = kMdRows * PS;
            const float *gp = part + (grp * kWarpsPerGroup) * ws;
            for (int e = gl; e < kMdRows * 8 * CH; e += kWarpsPerGroup * 32) {
                const int col = e / kMdRows, row = e - col * kMdRows;   // consecutive threads: consecutive rows
                const int j = 8 * c0 + col;
                if (row < st.nrows && j < n) {
                    const int o = row * PS + col;
                    float v = __fadd_rn(__fadd_rn(__fadd_rn(gp[o], gp[o + ws]), gp[o + 2 * ws]), gp[o + 3 * ws]);
                    if (KIND == 0 && pv.type == T_IQ2_S) v *= 0.125f;
                    if (KIND == 1) v = __fmul_rn(v, post);
                    p.out[(size_t)(sh.slot0[t] + j) * d_out + st.row0 + row] = v;
                }
            }
            group_sync(grp);   // the partial tiles are free again
            MDTRACE(it, 3);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }
}

// cb -> (tile, block within the tile) for the image kernels: every CTA scans the tiles' column blocks
__device__ int md_find_cb(const PfTile *tiles, int nt, int cb, int &cbi, int32_t *s_cnt) {
    // s_cnt: [kMdMaxTiles + 1] shared scratch; blockDim.x >= 256 threads
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    __shared__ int32_t wsum[32];
    __shared__ int32_t found;
    if (tid == 0) found = -1;
    __syncthreads();
    int carry = 0;
    for (int base = 0; base < nt; base += blockDim.x) {
        const int t = base + tid;
        const int c = t < nt ? (tiles[t].n + 7) / 8 : 0;
        int ci = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, ci, o);
            if (lane >= o) ci += a;
        }
        if (lane == 31) wsum[warp] = ci;
        __syncthreads();
        int pre = carry;
        for (int w = 0; w < warp; ++w) pre += wsum[w];
        if (t < nt && cb >= pre + ci - c && cb < pre + ci) { found = t; s_cnt[0] = cb - (pre + ci - c); }
        int tot = 0;
        for (int w = 0; w < nw; ++w) tot += wsum[w];
        __syncthreads();
        carry += tot;
    }
    __syncthreads();
    cbi = s_cnt[0];
    return found;
}

// gate_up operand image: CTA (cb, super-block); lane (g, c) of each warp-slice gets the q8 words of
// pair g of the block at K 64 i + {4c, 16 + 4c, 32 + 4c, 48 + 4c} (i = 0..3, the low / high nibble
// sub-blocks of Q4_K's 32-byte chunk i; IQ2_S's sub-blocks 2i, 2i + 1), the min-term word of the
// pair's bsums and the Q8_K scales of pairs 2c and 2c + 1. Absent pairs are zero.
__global__ void __launch_bounds__(256) md_bimg_kernel(const PfTile *tiles, const int32_t *n_tiles, const int32_t *perm,
                                                      const int8_t *xq8, const float *xd, const int16_t *xbs,
                                                      uint8_t *img, int k, int d) {
    __shared__ int32_t s_cnt[1];
    pdl_wait();
    pdl_launch_dependents();
    const int nsb = d / QK_K, cb = blockIdx.x, sb = blockIdx.y;
    int cbi = 0;
    const int t = md_find_cb(tiles, min(*n_tiles, kMdMaxTiles), cb, cbi, s_cnt);
    if (t < 0) return;
    const PfTile tl = tiles[t];
    const int tid = threadIdx.x, lane = tid & 31, part = tid >> 5;   // part 0..3: q8 words of chunk i; 4: min term
    if (part > 4) return;
    const int g = lane >> 2, c = lane & 3;
    uint8_t *dst = img + (size_t)cb * nsb * kMdGuSbBytes + (size_t)sb * kMdGuSbBytes + part * 512 + lane * 16;
    auto tok_of = [&](int col) { return 8 * cbi + col < tl.n ? perm[tl.slot0 + 8 * cbi + col] / k : -1; };
    if (part < 4) {
        const int tg = tok_of(g);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (tg >= 0) {
            const int8_t *q = xq8 + (size_t)tg * d + sb * QK_K + 64 * part + 4 * c;
            v.x = *reinterpret_cast<const uint32_t *>(q);
            v.y = *reinterpret_cast<const uint32_t *>(q + 16);
            v.z = *reinterpret_cast<const uint32_t *>(q + 32);
            v.w = *reinterpret_cast<const uint32_t *>(q + 48);
        }
        *reinterpret_cast<uint4 *>(dst) = v;
    } else {
        const int tg = tok_of(g), ta = tok_of(2 * c), tb = tok_of(2 * c + 1);
        uint32_t bw = 0u;
        if (tg >= 0) {
            const int16_t *bq = xbs + ((size_t)tg * nsb + sb) * 16 + 8 * (c & 1);
            const int p0 = bq[0] + bq[1], p1 = bq[2] + bq[3], p2 = bq[4] + bq[5], p3 = bq[6] + bq[7];
            bw = c < 2 ? pack_s8x4(p0 >> 6, p1 >> 6, p2 >> 6, p3 >> 6) : pack_s8x4(p0 & 63, p1 & 63, p2 & 63, p3 & 63);
        }
        const float dxa = ta >= 0 ? xd[(size_t)ta * nsb + sb] : 0.f, dxb = tb >= 0 ? xd[(size_t)tb * nsb + sb] : 0.f;
        *reinterpret_cast<uint4 *>(dst) = make_uint4(bw, __float_as_uint(dxa), __float_as_uint(dxb), 0u);
    }
}

// down operand image: CTA (cb, group of 8 32-blocks), one warp per 32-block b; lane (g, c): GeGLU of
// pair g's gate/up rows at K 32 b + {4c .. 4c + 3, 16 + 4c .. 16 + 4c + 3}, Q8_0 over the block's 32
// values (quantize_row_q8_0, arch/x86/quants.c:302: d = f16(amax / 127), q = rne(x * 127 / amax)),
// stored as {q words, d of pairs 2c, 2c + 1}. Optionally the pair-order gate_up rows for the caller.
__global__ void __launch_bounds__(256) md_act_kernel(const PfTile *tiles, const int32_t *n_tiles, const int32_t *perm,
                                                     const float *hbuf, uint8_t *img, float *h_pairs, int nff) {
    __shared__ int32_t s_cnt[1];
    pdl_wait();
    pdl_launch_dependents();
    const int nb = nff / QK32, cb = blockIdx.x;
    int cbi = 0;
    const int t = md_find_cb(tiles, min(*n_tiles, kMdMaxTiles), cb, cbi, s_cnt);
    if (t < 0) return;
    const PfTile tl = tiles[t];
    const int lane = threadIdx.x & 31, b = blockIdx.y * 8 + (threadIdx.x >> 5);
    if (b >= nb) return;
    const int g = lane >> 2, c = lane & 3;
    const bool valid = 8 * cbi + g < tl.n;
    const int slot = tl.slot0 + 8 * cbi + g;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (valid) {
        const float *hp = hbuf + (size_t)slot * 2 * nff + QK32 * b;
        const float4 ga = *reinterpret_cast<const float4 *>(hp + 4 * c), gb = *reinterpret_cast<const float4 *>(hp + 16 + 4 * c);
        const float4 ua = *reinterpret_cast<const float4 *>(hp + nff + 4 * c);
        const float4 ub = *reinterpret_cast<const float4 *>(hp + nff + 16 + 4 * c);
        v[0] = geglu1(ga.x, ua.x); v[1] = geglu1(ga.y, ua.y); v[2] = geglu1(ga.z, ua.z); v[3] = geglu1(ga.w, ua.w);
        v[4] = geglu1(gb.x, ub.x); v[5] = geglu1(gb.y, ub.y); v[6] = geglu1(gb.z, ub.z); v[7] = geglu1(gb.w, ub.w);
        if (h_pairs) {
            float *hq = h_pairs + (size_t)perm[slot] * 2 * nff + QK32 * b;
            *reinterpret_cast<float4 *>(hq + 4 * c) = ga;
            *reinterpret_cast<float4 *>(hq + 16 + 4 * c) = gb;
            *reinterpret_cast<float4 *>(hq + nff + 4 * c) = ua;
            *reinterpret_cast<float4 *>(hq + nff + 16 + 4 * c) = ub;
        }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float dd = h2f(f2h_rn(__fdiv_rn(amax, 127.f)));
    const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    int q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __float2int_rn(__fmul_rn(v[i], id));
    const float dxa = __shfl_sync(0xffffffffu, dd, 8 * c), dxb = __shfl_sync(0xffffffffu, dd, 8 * c + 4);
    uint8_t *dst = img + (size_t)cb * nb * kMdDnBlkBytes + (size_t)b * kMdDnBlkBytes + lane * 16;
    *reinterpret_cast<uint4 *>(dst) = make_uint4(pack_s8x4(q[0], q[1], q[2], q[3]), pack_s8x4(q[4], q[5], q[6], q[7]),
                                                 __float_as_uint(dxa), __float_as_uint(dxb));
}

static_assert(QK_K == 256 && QK32 == 32 && kMdGuSbBytes == 5 * 512 && kMdDnBlkBytes == 512,
              "md_image_bytes (params.h) sizes the images with these constants");

}  // namespace moeb
