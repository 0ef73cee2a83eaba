// MoE-FFN layer kernels for sm_100a (the library's single device translation unit).
//
//   fused_decode_kernel : the whole layer for up to 8 tokens in ONE persistent cooperative launch:
//                         router logits, routing (softmax / top-k / weights) and dispatch
//                         (histogram, exclusive scan, stable permutation), then the grouped
//                         gate_up and down GEMVs streamed HBM -> shared memory by bulk async copies
//                         and decoded in registers into integer dp4a dot products (the integer work
//                         of ggml-cpu's vec_dot kernels), and the slot-ordered combine.
//   gemv_kernel         : one projection of the moert per-kind ABI (moert_ffn_moe): the same
//                         grouped GEMV with routes given by the caller.
//   route_only / dequant / quant_act kernels : the inspection entry points of moeb200.h.
#include <cuda.h>

#include "common.cuh"

#include <algorithm>
#include <cstring>
#include <atomic>
#include <mutex>

#include "moeb200.h"

namespace moeb {

// ------------------------------------------------------------------ activation layout
// Q8_K activations are stored split per token: qs[nsb][256] int8 | d[nsb] f32 | bsums[nsb][16] i16,
// so the 32-value slices a lane reads are 16-byte aligned. Same numbers as ggml's block_q8_K.
struct Q8KView {
    const int8_t *qs;
    const float *d;
    const int16_t *bs;
};
__device__ __forceinline__ Q8KView q8k_view(const uint8_t *row, int nsb) {
    Q8KView v;
    v.qs = reinterpret_cast<const int8_t *>(row);
    v.d = reinterpret_cast<const float *>(row + nsb * 256);
    v.bs = reinterpret_cast<const int16_t *>(row + nsb * 256 + nsb * 4);
    return v;
}

// Q8_K quantisation of one 256-value super-block by one warp (quantize_row_q8_K_ref,
// ggml-quants.c:2696): the signed value of largest magnitude (first one on ties) sets
// iscale = -127/max; q = min(127, rne(iscale*x)); d = 1/iscale; bsums over 16 values.
// q8k_quantize_warp takes the lane's 8 values (lane * 8 .. lane * 8 + 7) in registers;
// q8k_superblock_warp loads them, with w given as the normed (x * s) * w (the Gemma-4 expert input).
__device__ __forceinline__ void q8k_quantize_warp(float (&v)[8], int8_t *qs, float *d_out, int16_t *bs, int lane);
__device__ void q8k_superblock_warp(const float *x, int8_t *qs, float *d_out, int16_t *bs, int lane,
                                    float nscale = 1.f, const float *w = nullptr) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[lane * 8 + i];
    if (w) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], nscale), w[lane * 8 + i]);
    }
    q8k_quantize_warp(v, qs, d_out, bs, lane);
}
__device__ __forceinline__ void q8k_quantize_warp(float (&v)[8], int8_t *qs, float *d_out, int16_t *bs, int lane) {
    float amax = 0.f;
    int aidx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fabsf(v[i]);
        if (a > amax) { amax = a; aidx = lane * 8 + i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const int oi = __shfl_xor_sync(0xffffffffu, aidx, o);
        if (oa > amax || (oa == amax && oi < aidx)) { amax = oa; aidx = oi; }
    }
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) qs[lane * 8 + i] = 0;
        if ((lane & 1) == 0) bs[lane >> 1] = 0;
        if (lane == 0) *d_out = 0.f;
        return;
    }
    const float vmax = __shfl_sync(0xffffffffu, v[aidx & 7], aidx >> 3);
    const float iscale = __fdiv_rn(-127.f, vmax);
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int q = __float2int_rn(__fmul_rn(iscale, v[i]));
        q = q < 127 ? q : 127;
        qs[lane * 8 + i] = (int8_t)q;
        s += q;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if ((lane & 1) == 0) bs[lane >> 1] = (int16_t)s;
    if (lane == 0) *d_out = __fdiv_rn(1.f, iscale);
}

// ------------------------------------------------------------------ routing + dispatch in a CTA
struct RouteSmem {
    int32_t ids[kMaxPairs];
    float w[kMaxPairs];
    int32_t cnt[kMaxE];
    int32_t off[kMaxE + 1];
    int32_t perm[kMaxPairs];
    int32_t n_unique;
    int32_t uexp[kMaxPairs];      // unique routed experts, ascending
    int32_t ucls[kMaxPairs];      // 0 hot, 1 cold
    int32_t uwidx[kMaxPairs];     // index into the class pool (slot / expert)
    long long upre[kMaxPairs + 1];  // cumulative weight bytes
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

// softmax -> top-k (value desc, index asc) -> normalised weights, one warp per token
// (llama-graph.cpp:1553-1648; the reference's argsort is unstable, so ties go to the lowest id).
__device__ void route_tokens(const RouteSrc &r, RouteSmem &rs, int tid, int nwarps) {
    const int lane = tid & 31, warp = tid >> 5;
    const int per = r.E / 32;
    for (int t = warp; t < r.T; t += nwarps) {
        if (r.logits) {
            float v[kMaxE / 32];
#pragma unroll
            for (int i = 0; i < kMaxE / 32; ++i) v[i] = i < per ? r.logits[(size_t)t * r.E + lane + 32 * i] : -INFINITY;
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
            float psum = 0.f;
            for (int j = 0; j < r.k; ++j) {
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
                if (lane == 0) { rs.ids[t * r.k + j] = bi; rs.w[t * r.k + j] = pj; }
            }
            psum = fmaxf(psum, 6.103515625e-5f);
            __syncwarp();
            if (lane < r.k) rs.w[t * r.k + lane] = __fdiv_rn(rs.w[t * r.k + lane], psum);
        } else if (lane < r.k) {
            rs.ids[t * r.k + lane] = r.ids[(size_t)t * r.ids_s1 + lane];
            rs.w[t * r.k + lane] = 1.f;
        }
    }
}

// Histogram, exclusive scan and stable permutation of the routed pairs (the grouping of
// ggml-cpu's mul_mat_id, ggml-cpu.c:1613-1626), plus the unique-expert list with each expert's
// precision class and cumulative weight bytes for the work split.
__device__ void dispatch_pairs(const RouteSrc &r, const Residency &res, const PoolView &hot, const PoolView &cold,
                               int d_in, int d_out, RouteSmem &rs, int tid, int nthreads, bool check_pools) {
    const int P = r.T * r.k;
    for (int e = tid; e < r.E; e += nthreads) rs.cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += nthreads) {
        int e = rs.ids[p];
        if (e < 0 || e >= r.E) { atomicOr(&g_error, ERR_BAD_EXPERT); e = 0; rs.ids[p] = 0; }
        atomicAdd(&rs.cnt[e], 1);
    }
    __syncthreads();
    const int lane = tid & 31;
    if (tid < 32) {
        // exclusive scan of cnt over E (<= 256) and the unique-expert compaction, one warp
        int base = 0, ubase = 0;
        long long cbase = 0;
        for (int e0 = 0; e0 < r.E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < r.E ? rs.cnt[e] : 0;
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            if (e < r.E) rs.off[e] = base + incl - c;
            base += __shfl_sync(0xffffffffu, incl, 31);
            bool has = c > 0;
            long long cost = 0;
            int cls = 1, widx = e;
            if (has) {
                if (res.n_slots > 0 && res.exp_slot) {
                    const int s = res.exp_slot[e];
                    if (s >= 0 && s < res.n_slots && res.slot_state[s] == 2 && res.slot_exp[s] == e) { cls = 0; widx = s; }
                }
                const PoolView &pv = cls == 0 ? hot : cold;
                // an expert whose class pool is absent (or whose table entry is not 16-byte aligned)
                // is reported and left out of the work split instead of being read
                const bool ok = !check_pools ||
                                (pv.ptrs ? ((reinterpret_cast<uintptr_t>(pv.ptrs[widx]) & 15u) == 0 && pv.ptrs[widx])
                                         : (pv.w != nullptr && widx < pv.n));
                if (!ok) { atomicOr(&g_error, ERR_BAD_EXPERT); has = false; }
                cost = (long long)d_out * row_bytes(pv.type, d_in);
            }
            const unsigned m = __ballot_sync(0xffffffffu, has);
            if (!has) cost = 0;
            long long cincl = cost;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long n = __shfl_up_sync(0xffffffffu, cincl, o);
                if (lane >= o) cincl += n;
            }
            if (has) {
                const int u = ubase + __popc(m & ((1u << lane) - 1u));
                rs.uexp[u] = e;
                rs.ucls[u] = cls;
                rs.uwidx[u] = widx;
                rs.upre[u + 1] = cbase + cincl;
            }
            ubase += __popc(m);
            cbase += __shfl_sync(0xffffffffu, cincl, 31);
        }
        if (lane == 0) {
            rs.off[r.E] = base;
            rs.n_unique = ubase;
            rs.upre[0] = 0;
        }
    }
    __syncthreads();
    // stable rank of each pair within its expert (P <= 256: quadratic is cheaper than a sort)
    for (int p = tid; p < P; p += nthreads) {
        const int e = rs.ids[p];
        int rank = 0;
        for (int q = 0; q < p; ++q) rank += rs.ids[q] == e;
        rs.perm[rs.off[e] + rank] = p;
    }
    __syncthreads();
}

// ------------------------------------------------------------------ shared-memory word access
// Quantised blocks sit in shared memory at 2-byte aligned addresses (902-, 82-, 22- and 18-byte
// strides). Runs of 32-bit words are read with aligned 32-bit loads and realigned with a funnel
// shift; stage buffers carry 16 bytes of padding so the extra word read at the end stays inside.
template <int N>
__device__ __forceinline__ void lds_words_a2(const uint8_t *p, uint32_t (&w)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(a & 2u) * 8u;   // 0 or 16
    uint32_t raw[N + 1];
#pragma unroll
    for (int i = 0; i <= N; ++i) raw[i] = base[i];
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
}


// per-token activation rows in shared memory (pointers hoisted out of the block loops)
struct ActQ8K {           // Q8_K row split as qs[nsb][256] | d[nsb] f32 | bsums[nsb][16] i16
    const int8_t *qs;
    const float *d;
    const int16_t *bs;
};
struct ActQ80 {           // Q8_0 row split as qs[nb][32] | d[nb] f32 | qsum[nb] i32
    const int8_t *qs;
    const float *d;
    const int *qsum;
};

// ------------------------------------------------------------------ gate_up row dot products
// Eight threads share a row; thread L computes the reference's lane L of the x86 kernels
// (ggml_vec_dot_q4_K_q8_K, x86/quants.c:1900; _iq2_s_q8_K :2937; _iq2_xxs_q8_K :2522): the integer
// sum of the products at positions 4L..4L+3 of each 32-value group of a super-block (one dp4a per
// group, the group's scale inside the integer), fused-multiply-added into its own f32 chain with
// the super-block's d_x * d_w. gu_rows then adds the eight chains in the reference's order. Q4_K's
// min term: thread L also runs min lane m = L & 3, mins[2m] * q8s[2m] + mins[2m+1] * q8s[2m+1]
// (q8s = the 32-value sub-block sums), in a chain scaled by -d_x * dmin_w.

// Q4_K (rows 16-byte aligned): byte 32c + b of qs holds value b of sub-block 2c (low nibble) and of
// sub-block 2c + 1 (high nibble), so lane L's values of chunk c are the nibbles of one word
template <int NT>
__device__ __forceinline__ void q4k_lane(const uint8_t *row, int nsb, int L, const ActQ8K (&x)[NT], float (&acc)[NT],
                                         float (&macc)[NT]) {
    const int m = L & 3;
    const uint32_t M = 0x0f0f0f0fu;
#pragma unroll 1
    for (int sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + sb * B_Q4_K;
        const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);   // d, dmin | scales[12]
        const float dw = h2f((uint16_t)(hdr.x & 0xffffu)), dmin = h2f((uint16_t)(hdr.x >> 16));
        uint8_t sc12[12];
        *reinterpret_cast<uint32_t *>(sc12) = hdr.y;
        *reinterpret_cast<uint32_t *>(sc12 + 4) = hdr.z;
        *reinterpret_cast<uint32_t *>(sc12 + 8) = hdr.w;
        int sc[8], mn[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q4k_scale_min(j, sc12, sc[j], mn[j]);
        uint32_t qw[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) qw[c] = *reinterpret_cast<const uint32_t *>(blk + 16 + 32 * c + 4 * L);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int *q8 = reinterpret_cast<const int *>(x[t].qs + sb * 256);
            int sum = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                sum += sc[2 * c] * dp4a((int)(qw[c] & M), q8[16 * c + L], 0);
                sum += sc[2 * c + 1] * dp4a((int)((qw[c] >> 4) & M), q8[16 * c + 8 + L], 0);
            }
            const float yd = x[t].d[sb];
            acc[t] = fmaf(__fmul_rn(yd, dw), (float)sum, acc[t]);
            const int16_t *bs = x[t].bs + sb * 16 + 4 * m;
            const int msum = mn[2 * m] * ((int)bs[0] + (int)bs[1]) + mn[2 * m + 1] * ((int)bs[2] + (int)bs[3]);
            macc[t] = fmaf(-__fmul_rn(yd, dmin), (float)msum, macc[t]);
        }
    }
}

// IQ2_S (82-byte blocks, 2-byte aligned): value 32b + 4L + e is byte 4(L & 1) + e of grid entry
// g = 4b + L/2, negated where bit 4(L & 1) + e of signs[g] is set, times 2 * (L < 4 ? low : high
// scale nibble of block b) + 1; the caller scales the total by 1/8
template <int NT>
__device__ __forceinline__ void iq2s_lane(const uint8_t *row, int nsb, int L, const uint64_t *grid,
                                          const ActQ8K (&x)[NT], float (&acc)[NT]) {
#pragma unroll 1
    for (int sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + sb * B_IQ2_S;
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(blk));
        int wv[8], ls[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int g = 4 * b + (L >> 1);
            const uint32_t gi = (uint32_t)blk[2 + g] | ((((uint32_t)blk[66 + b] >> (2 * (g & 3))) & 3u) << 8);
            const uint32_t mag = (uint32_t)(grid[gi] >> (32 * (L & 1)));
            const uint32_t c = ((((uint32_t)blk[34 + g] >> (4 * (L & 1))) & 15u) * 0x00204081u) & 0x01010101u;
            // negate flagged bytes: (w ^ 0xff) + 1 == -w; magnitudes are >= 8, so nothing carries
            wv[b] = (int)((mag ^ (c * 0xffu)) + c);
            const uint32_t sv = blk[74 + b];
            ls[b] = 2 * (int)(L < 4 ? (sv & 15u) : (sv >> 4)) + 1;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int *q8 = reinterpret_cast<const int *>(x[t].qs + sb * 256);
            int sum = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) sum += ls[b] * dp4a(wv[b], q8[8 * b + L], 0);
            acc[t] = fmaf(__fmul_rn(dw, x[t].d[sb]), (float)sum, acc[t]);
        }
    }
}

// IQ2_XXS (66-byte blocks, 2-byte aligned): per 32-block b, 4 grid indices then a word of four 7-bit
// sign-pattern indices and a 4-bit scale; value 32b + 4L + e is byte 4(L & 1) + e of grid entry
// aux[L/2], signed by that pattern, times 2 * ls + 1; the caller scales the total by 1/8
template <int NT>
__device__ __forceinline__ void iq2xxs_lane(const uint8_t *row, int nsb, int L, const ActQ8K (&x)[NT], float (&acc)[NT]) {
    const int l = L >> 1;
#pragma unroll 1
    for (int sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + sb * B_IQ2_XXS;
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(blk));
        int wv[8], ls[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const uint8_t *g8 = blk + 2 + 8 * b;
            const uint32_t hi = (uint32_t)*reinterpret_cast<const uint16_t *>(g8 + 4) |
                                ((uint32_t)*reinterpret_cast<const uint16_t *>(g8 + 6) << 16);
            const uint32_t mag = (uint32_t)(g_iq2xxs_grid[g8[l]] >> (32 * (L & 1)));
            const uint32_t c = ((((uint32_t)g_iq2xxs_signs[(hi >> (7 * l)) & 127u] >> (4 * (L & 1))) & 15u) * 0x00204081u) &
                               0x01010101u;
            wv[b] = (int)((mag ^ (c * 0xffu)) + c);
            ls[b] = 2 * (int)(hi >> 28) + 1;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int *q8 = reinterpret_cast<const int *>(x[t].qs + sb * 256);
            int sum = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) sum += ls[b] * dp4a(wv[b], q8[8 * b + L], 0);
            acc[t] = fmaf(__fmul_rn(dw, x[t].d[sb]), (float)sum, acc[t]);
        }
    }
}

// ---------------------------------------------------------------- warp-level int8 MMA helpers
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &d0, uint32_t &d1, uint32_t &d2, uint32_t &d3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
                 : "r"(addr)
                 : "memory");
}
// D = A (16x32 s8, row) * B (32x8 s8, col), exact int32
__device__ __forceinline__ void mma_s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1) {
    d[0] = d[1] = d[2] = d[3] = 0;
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    d[0] = d[1] = d[2] = d[3] = 0;
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xffu); }
__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)(d & 0xff) << 24);
}

// Q5_0 x Q8_0, lane = half of a row's 32-blocks: value = (nibble | hbit << 4) - 16, so
// dot = sum(u * q) - 16 * sum(q); d_w * d_x per block.
template <int NT>
__device__ __forceinline__ void q5_0_lane(const uint8_t *row, int b0, int b1, const ActQ80 (&x)[NT], float (&acc)[NT]) {
#pragma unroll 1
    for (int b = b0; b < b1; ++b) {
        const uint8_t *blk = row + b * B_Q5_0;
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(blk));
        uint32_t w[5];                                  // qh | qs[0..15]
        lds_words_a2<5>(blk + 2, w);
        const uint32_t qh = w[0];
        int wlo[4], whi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t hl = (((qh >> (4 * i)) & 15u) * 0x00204081u) & 0x01010101u;
            const uint32_t hh = (((qh >> (16 + 4 * i)) & 15u) * 0x00204081u) & 0x01010101u;
            wlo[i] = (int)((w[1 + i] & 0x0f0f0f0fu) | (hl << 4));
            whi[i] = (int)(((w[1 + i] >> 4) & 0x0f0f0f0fu) | (hh << 4));
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int4 *q = reinterpret_cast<const int4 *>(x[t].qs + 32 * b);
            const int4 xa = q[0], xb = q[1];
            int s = dp4a(wlo[0], xa.x, 0);
            s = dp4a(wlo[1], xa.y, s);
            s = dp4a(wlo[2], xa.z, s);
            s = dp4a(wlo[3], xa.w, s);
            s = dp4a(whi[0], xb.x, s);
            s = dp4a(whi[1], xb.y, s);
            s = dp4a(whi[2], xb.z, s);
            s = dp4a(whi[3], xb.w, s);
            s -= 16 * x[t].qsum[b];
            acc[t] = fmaf(dw * x[t].d[b], (float)s, acc[t]);
        }
    }
}

// 4 IQ4_NL level lookups for the low nibbles of the 4 bytes of w (levels packed in t0..t3)
__device__ __forceinline__ int iq4nl_lookup4(uint32_t w, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3) {
    const uint32_t x = w & 0x0f0f0f0fu;
    const uint32_t y = x | (x >> 4);
    const uint32_t sel = (y & 0xffu) | ((y >> 8) & 0xff00u);
    const uint32_t lo = __byte_perm(t0, t1, sel & 0x7777u);
    const uint32_t hi = __byte_perm(t2, t3, sel & 0x7777u);
    const uint32_t m = ((x >> 3) & 0x01010101u) * 0xffu;
    return (int)((lo & ~m) | (hi & m));
}

// IQ4_NL x Q8_0, lane = half of a row's 32-blocks
template <int NT>
__device__ __forceinline__ void iq4nl_lane(const uint8_t *row, int b0, int b1, const ActQ80 (&x)[NT],
                                           const uint32_t (&kv)[4], float (&acc)[NT]) {
#pragma unroll 1
    for (int b = b0; b < b1; ++b) {
        const uint8_t *blk = row + b * B_IQ4_NL;
        const float dw = h2f(*reinterpret_cast<const uint16_t *>(blk));
        uint32_t w[4];
        lds_words_a2<4>(blk + 2, w);
        int wlo[4], whi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wlo[i] = iq4nl_lookup4(w[i], kv[0], kv[1], kv[2], kv[3]);
            whi[i] = iq4nl_lookup4(w[i] >> 4, kv[0], kv[1], kv[2], kv[3]);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const int4 *q = reinterpret_cast<const int4 *>(x[t].qs + 32 * b);
            const int4 xa = q[0], xb = q[1];
            int s = dp4a(wlo[0], xa.x, 0);
            s = dp4a(wlo[1], xa.y, s);
            s = dp4a(wlo[2], xa.z, s);
            s = dp4a(wlo[3], xa.w, s);
            s = dp4a(whi[0], xb.x, s);
            s = dp4a(whi[1], xb.y, s);
            s = dp4a(whi[2], xb.z, s);
            s = dp4a(whi[3], xb.w, s);
            acc[t] = fmaf(x[t].d[b] * dw, (float)s, acc[t]);
        }
    }
}

// ------------------------------------------------------------------ Q8_0 activations for down
// One warp quantises one 32-block: AVX2 semantics of quantize_row_q8_0 (arch/x86/quants.c:302):
// d = f16(amax / 127), q = rne(x * (127 / amax)); also keeps sum(q) for the Q5_0 offset.
__device__ __forceinline__ void q80_block_warp(float v, int8_t *qs, float *d, int *qsum, int lane) {
    const float amax = warp_max(fabsf(v));
    const float dd = h2f(f2h_rn(__fdiv_rn(amax, 127.f)));
    const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
    const int q = __float2int_rn(__fmul_rn(v, id));
    qs[lane] = (int8_t)q;
    int s = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) { *d = dd; *qsum = s; }
}

// GeGLU with ggml-cpu's fp16-table GELU (ggml-cpu/vec.h:1414-1430)
__device__ __forceinline__ float geglu1(float g, float u) {
    if (g <= -10.0f) return 0.0f;
    if (g >= 10.0f) return __fmul_rn(g, u);
    return __fmul_rn(h2f(g_gelu_f16[f2h_rn(g)]), u);
}

// ------------------------------------------------------------------ the grouped GEMV
// One CTA per SM: a producer warp streams stages of weight rows HBM -> shared memory with bulk
// copies; 16 consumer warps in 4 groups take every 4th stage. Each stage slot has a `full`
// barrier (copy landed) and an `empty` barrier (its group's 4 warps are done), so groups never
// wait for one another, only for data.
constexpr int kConsumerWarps = 16;
constexpr int kGroups = 4;
constexpr int kWarpsPerGroup = kConsumerWarps / kGroups;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kSlots = 6;
constexpr int kGuStageRows = kWarpsPerGroup * 4;    // 8 lanes per row, 4 rows per warp
constexpr int kDnStageRows = kWarpsPerGroup * 16;   // 2 lanes per row, 16 rows per warp

struct GemvSmem {
    int route, bars, grid, act, stage, stage_cap, total;
};
__host__ __device__ inline GemvSmem gemv_layout(int kind, int d_in, int T) {
    GemvSmem L;
    int o = 0;
    L.route = o; o += (int)((sizeof(RouteSmem) + 127) / 128 * 128);
    L.bars = o;  o += (2 * kSlots * 8 + 127) / 128 * 128;
    L.grid = o;  o += kind == 0 ? MOE_IQ2S_GRID_ROWS * 8 : 0;
    L.act = o;   o += kind == 0 ? T * xq_stride_bytes(d_in) : 2 * T * q80_stride(d_in);
    o = (o + 127) / 128 * 128;
    L.stage = o;
    const int rows = kind == 0 ? kGuStageRows : kDnStageRows;
    const int rb = kind == 0 ? (int)row_bytes(T_Q4_K, d_in) : (int)row_bytes(T_Q5_0, d_in);
    L.stage_cap = (rows * rb + 16 + 127) / 128 * 128;
    o += kSlots * L.stage_cap;
    L.total = o;
    return L;
}

__device__ __forceinline__ const uint8_t *pool_entry(const PoolView &pv, int widx, int d_out, int d_in) {
    if (pv.ptrs) return reinterpret_cast<const uint8_t *>(pv.ptrs[widx]);
    return pv.w + (size_t)widx * d_out * row_bytes(pv.type, d_in);
}

// flat group index (8-row groups; every unique expert has gpe groups) of byte position `pos`
__device__ __forceinline__ int group_at(const RouteSmem &rs, long long pos, int gpe) {
    const int U = rs.n_unique;
    if (pos >= rs.upre[U]) return U * gpe;
    int lo = 0, hi = U - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (rs.upre[mid] <= pos) lo = mid; else hi = mid - 1;
    }
    const long long per = (rs.upre[lo + 1] - rs.upre[lo]) / gpe;
    return lo * gpe + (int)((pos - rs.upre[lo]) / per);
}

// Stages never cross an expert and sit on a per-expert grid of `sg` groups, so stage s of the CTA
// range [g0, g1) is computable from s alone.
struct StagePlan {
    int u, row0, nrows;
};
__device__ __forceinline__ int stage_of(int g, int gpe, int spe, int sg) { return (g / gpe) * spe + (g % gpe) / sg; }
__device__ __forceinline__ StagePlan stage_plan(int s, int g0, int g1, int gpe, int spe, int sg) {
    StagePlan p;
    p.u = s / spe;
    const int k = s - p.u * spe;
    const int base = p.u * gpe;
    const int lo = max(base + k * sg, g0);
    const int hi = min(min(base + (k + 1) * sg, base + gpe), g1);
    p.row0 = (lo - base) * kGroupRows;
    p.nrows = (hi - lo) * kGroupRows;
    return p;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// the four warps of consumer group g (named barriers 2 .. 5)
__device__ __forceinline__ void group_sync(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(2 + g), "r"(kWarpsPerGroup * 32) : "memory");
}
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
}

template <int NT>
__device__ __forceinline__ void gu_rows(const uint8_t *row, int nsb, int j, int type, const uint64_t *grid,
                                        const uint8_t *act, int xs, const int *tok, float (&out)[4]) {
    ActQ8K x[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint8_t *a = act + (size_t)tok[t] * xs;
        x[t].qs = reinterpret_cast<const int8_t *>(a);
        x[t].d = reinterpret_cast<const float *>(a + nsb * 256);
        x[t].bs = reinterpret_cast<const int16_t *>(a + nsb * 256 + nsb * 4);
    }
    float acc[NT], macc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = macc[t] = 0.f;
    if (type == T_IQ2_S) iq2s_lane<NT>(row, nsb, j, grid, x, acc);
    else if (type == T_IQ2_XXS) iq2xxs_lane<NT>(row, nsb, j, x, acc);
    else q4k_lane<NT>(row, nsb, j, x, acc, macc);
    // the reference's reductions (hsum_float_8: ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)); the
    // min lanes (m0 + m2) + (m1 + m3), added last); every thread of the row ends with the same value
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        float s = acc[t];
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 4));
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
        if (type == T_Q4_K) {
            float m = macc[t];
            m = __fadd_rn(m, __shfl_xor_sync(0xffffffffu, m, 2));
            m = __fadd_rn(m, __shfl_xor_sync(0xffffffffu, m, 1));
            s = __fadd_rn(s, m);
        } else {
            s = __fmul_rn(0.125f, s);
        }
        out[t] = s;
    }
}

template <int NT>
__device__ __forceinline__ void dn_rows(const uint8_t *row, int b0, int b1, int nb, int type, const uint32_t (&kv)[4],
                                        const uint8_t *act, int as, int slot0, int nt, float (&out)[4]) {
    ActQ80 x[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const uint8_t *a = act + (size_t)(slot0 + (t < nt ? t : 0)) * as;   // missing columns repeat column 0
        x[t].qs = reinterpret_cast<const int8_t *>(a);
        x[t].d = reinterpret_cast<const float *>(a + nb * 32);
        x[t].qsum = reinterpret_cast<const int *>(a + nb * 36);
    }
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.f;
    if (type == T_Q5_0) q5_0_lane<NT>(row, b0, b1, x, acc);
    else iq4nl_lane<NT>(row, b0, b1, x, kv, acc);
#pragma unroll
    for (int t = 0; t < NT; ++t) out[t] = acc[t];
}

#ifdef MOEB_TRACE
__device__ unsigned long long g_trace[2][512][8];
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define TRACE(i) do { if ((threadIdx.x & 31) == 0 && blockIdx.x < 512) g_trace[p.kind == 0 ? 0 : 1][blockIdx.x][i] = gtime(); } while (0)
#define FTRACE(i) do { if ((threadIdx.x & 31) == 0 && blockIdx.x < 512) g_ftrace[blockIdx.x][i] = clock64(); } while (0)
__device__ unsigned long long g_ftrace[512][16];
__device__ unsigned long long g_strace[512][64][3];   // per stage of warp 0: start, data ready, done
#else
#define TRACE(i) do { } while (0)
#define FTRACE(i) do { } while (0)
#endif
#ifdef MOEB_TRACE
#define STRACE(it, k) do { if (warp == 0 && lane == 0 && blockIdx.x < 512 && (it) < 64) g_strace[blockIdx.x][(it)][k] = clock64(); } while (0)
#else
#define STRACE(it, k) do { } while (0)
#endif

__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GemvSmem L = gemv_layout(p.kind == 0 ? 0 : 1, p.d_in, p.route.T);
    RouteSmem &rs = *reinterpret_cast<RouteSmem *>(smem + L.route);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + kSlots;
    uint64_t *grid = reinterpret_cast<uint64_t *>(smem + L.grid);
    uint8_t *act = smem + L.act;
    uint8_t *stage = smem + L.stage;

    // ---- prologue independent of upstream results
    if (tid == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarpsPerGroup);
        }
        fence_mbar_init();
    }
    if (p.kind == 0)
        for (int i = tid; i < MOE_IQ2S_GRID_ROWS; i += kGemvThreads) grid[i] = g_iq2s_grid[i];
    uint32_t kv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        kv[i] = (uint32_t)(uint8_t)g_iq4nl[4 * i] | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 1] << 8) |
                ((uint32_t)(uint8_t)g_iq4nl[4 * i + 2] << 16) | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 3] << 24);

    // gate_up reads the router's logits and activations: wait for the router grid. The down
    // projection's routing inputs were complete before the gate_up grid got past its own wait, so
    // it routes and starts streaming weights first and waits for the gate_up outputs later.
    if (warp == 0) TRACE(0);
    if (p.kind == 0) pdl_wait();
    __syncthreads();
    if (warp == 0) TRACE(1);

    // ---- routing and dispatch (every CTA, identical results)
    route_tokens(p.route, rs, tid, kGemvThreads / 32);
    __syncthreads();
    if (warp == 0) TRACE(2);
    dispatch_pairs(p.route, p.res, p.hot, p.cold, p.d_in, p.d_out, rs, tid, kGemvThreads, true);
    if (warp == 0) TRACE(3);
    const int T = p.route.T, k = p.route.k, P = T * k;
    if (blockIdx.x == 0) {
        for (int i = tid; i < P; i += kGemvThreads) {
            if (p.ids_out) p.ids_out[i] = rs.ids[i];
            if (p.w_out) p.w_out[i] = rs.w[i];
            if (p.perm_out) p.perm_out[i] = rs.perm[i];
        }
        for (int e = tid; e <= p.route.E; e += kGemvThreads) {
            if (p.cnt_out && e < p.route.E) p.cnt_out[e] = rs.cnt[e];
            if (p.off_out) p.off_out[e] = rs.off[e];
            if (p.rc_counts && e < p.route.E && rs.cnt[e]) atomicAdd(&p.rc_counts[e], rs.cnt[e]);
        }
        if (p.rc_hits && tid < rs.n_unique) {
            const int e = rs.uexp[tid];
            atomicAdd(&p.rc_hits[rs.ucls[tid] == 0 ? 0 : 1], rs.cnt[e]);
        }
    }
    pdl_launch_dependents();

    // ---- this CTA's share of the routed experts' weight bytes, in 8-row groups and stages
    const int gpe = p.d_out / kGroupRows;
    const int sg = (p.kind == 0 ? kGuStageRows : kDnStageRows) / kGroupRows;
    const int spe = (gpe + sg - 1) / sg;
    const long long total = rs.upre[rs.n_unique];
    const long long s0 = total * blockIdx.x / gridDim.x, s1 = total * (blockIdx.x + 1) / gridDim.x;
    const int g0 = group_at(rs, s0, gpe), g1 = group_at(rs, s1, gpe);
    if (g0 >= g1) return;   // no barrier below involves a CTA without work
    const int S0 = stage_of(g0, gpe, spe, sg);
    const int n_st = stage_of(g1 - 1, gpe, spe, sg) - S0 + 1;

    if (warp == kConsumerWarps) {
        // ---- producer: one lane streams the stages through the slot ring
        if (lane == 0) {
            TRACE(4);
            for (int it = 0; it < n_st; ++it) {
                const int slot = it % kSlots;
                if (it >= kSlots && !mbar_wait(&empty[slot], (uint32_t)(((it / kSlots) - 1) & 1))) break;
                const StagePlan st = stage_plan(S0 + it, g0, g1, gpe, spe, sg);
                const PoolView &pv = rs.ucls[st.u] == 0 ? p.hot : p.cold;
                const int rb = (int)row_bytes(pv.type, p.d_in);
                const uint32_t bytes = (uint32_t)(st.nrows * rb);
                mbar_expect_tx(&full[slot], bytes);
                bulk_g2s(stage + slot * L.stage_cap,
                         pool_entry(pv, rs.uwidx[st.u], p.d_out, p.d_in) + (size_t)st.row0 * rb, bytes, &full[slot]);
            }
        }
        return;
    }

    // ---- consumers: activations for this CTA's experts
    const int nsb = p.d_in / QK_K, nb = p.d_in / QK32;
    const int u_first = g0 / gpe;
    if (p.kind == 0) {
        const int n16 = T * p.xq_stride / 16;
        const int4 *src = reinterpret_cast<const int4 *>(p.xq);
        int4 *dst = reinterpret_cast<int4 *>(act);
        for (int i = tid; i < n16; i += kConsumerWarps * 32) dst[i] = src[i];
    } else {
        if (p.kind == 1) pdl_wait();   // gate_up outputs
        const int as = q80_stride(p.d_in);
        const int u_last = (g1 - 1) / gpe;
        if (u_last - u_first > 1 && tid == 0) atomicOr(&g_error, ERR_CAPACITY);
        for (int u = u_first; u <= min(u_last, u_first + 1); ++u) {
            const int e = rs.uexp[u], po = rs.off[e], n = min(rs.cnt[e], T);
            for (int item = warp; item < n * nb; item += kConsumerWarps) {
                const int i = item / nb, b = item - i * nb;
                const int pair = rs.perm[po + i];
                float v;
                if (p.kind == 1) {
                    const float *hp = p.h + (size_t)pair * 2 * p.d_in;
                    v = geglu1(hp[32 * b + lane], hp[p.d_in + 32 * b + lane]);
                } else {
                    v = p.a[(size_t)(p.a_per_pair ? pair : pair / k) * p.d_in + 32 * b + lane];
                }
                uint8_t *row = act + (size_t)((u - u_first) * T + i) * as;
                q80_block_warp(v, reinterpret_cast<int8_t *>(row) + 32 * b, reinterpret_cast<float *>(row + nb * 32) + b,
                               reinterpret_cast<int *>(row + nb * 36) + b, lane);
            }
        }
    }
    consumer_sync();
    if (warp == 0) TRACE(5);

    // ---- consumers: stages
    const int grp = warp / kWarpsPerGroup, wg = warp % kWarpsPerGroup;
    const int xs = p.xq_stride, as = q80_stride(p.d_in);
    for (int it = grp; it < n_st; it += kGroups) {
        const int slot = it % kSlots;
        if (!mbar_wait(&full[slot], (uint32_t)((it / kSlots) & 1))) break;
        const StagePlan st = stage_plan(S0 + it, g0, g1, gpe, spe, sg);
        const int e = rs.uexp[st.u], cls = rs.ucls[st.u], widx = rs.uwidx[st.u];
        const int po = rs.off[e];
        const PoolView &pv = cls == 0 ? p.hot : p.cold;
        const int rb = (int)row_bytes(pv.type, p.d_in);
        const uint8_t *sbuf = stage + slot * L.stage_cap;
        if (p.kind == 0) {
            const int n = rs.cnt[e];
            const int j = lane & 7, r = wg * 4 + (lane >> 3);
            if (wg * 4 < st.nrows) {
                const uint8_t *row = sbuf + (size_t)r * rb;
                for (int c0 = 0; c0 < n; c0 += kTokChunk) {
                    const int nt = min(kTokChunk, n - c0);
                    int tok[kTokChunk], pair[kTokChunk];
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        pair[c] = rs.perm[po + c0 + (c < nt ? c : 0)];
                        tok[c] = pair[c] / k;
                    }
                    float v[4] = {0.f, 0.f, 0.f, 0.f};
                    if (nt == 1) gu_rows<1>(row, nsb, j, pv.type, grid, act, xs, tok, v);
                    else gu_rows<4>(row, nsb, j, pv.type, grid, act, xs, tok, v);
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c)
                        if (j == 0 && c < nt) p.y[(size_t)pair[c] * p.d_out + st.row0 + r] = v[c];
                }
            }
        } else {
            int n = rs.cnt[e];
            if (n > T) {
                // the activation buffer holds one pair per token of an expert; an expert repeated
                // within a token's routes is reported and its extra pairs are not computed
                if (lane == 0) atomicOr(&g_error, ERR_CAPACITY);
                n = T;
            }
            const int half = lane & 1, r = wg * 16 + (lane >> 1);
            const int bmid = (nb + 1) / 2, b0 = half ? bmid : 0, b1 = half ? nb : bmid;
            const bool valid = r < st.nrows;
            const int slot0 = (st.u - u_first) * T;
            if (wg * 16 < st.nrows) {
                const uint8_t *row = sbuf + (size_t)(valid ? r : 0) * rb;
                for (int c0 = 0; c0 < n; c0 += kTokChunk) {
                    const int nt = min(kTokChunk, n - c0);
                    float v[4] = {0.f, 0.f, 0.f, 0.f};
                    if (nt == 1) dn_rows<1>(row, b0, b1, nb, pv.type, kv, act, as, slot0 + c0, nt, v);
                    else dn_rows<4>(row, b0, b1, nb, pv.type, kv, act, as, slot0 + c0, nt, v);
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        float s = v[c];
                        s += __shfl_xor_sync(0xffffffffu, s, 1);
                        if (half == 0 && valid && c < nt) {
                            const int pair = rs.perm[po + c0 + c];
                            if (p.apply_scale && pv.scale) s = __fmul_rn(s, pv.scale[widx]);
                            p.y[(size_t)pair * p.d_out + st.row0 + r] = s;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (warp == 0 && it == 0) TRACE(6);
    }
    if (warp == 0) TRACE(7);
}

// ------------------------------------------------------------------ fused decode layer
// The whole layer for up to kFusedMaxT tokens in ONE persistent cooperative kernel (one CTA per
// SM), phases separated by bounded grid barriers:
//   A  router logits (one CTA per expert, fixed-order reduction) + bias; Q8_K of every token;
//      every CTA also loads the residency class of every expert and the IQ2_S codebook
//   -- grid barrier 1 --
//   B  every CTA: softmax / top-k / weights and the dispatch (histogram, scan, stable
//      permutation), then its byte-balanced share of the routed experts' gate_up AND down rows;
//      the producer warp streams the gate_up stages and then, without a break, the down stages
//      through one ring of shared-memory slots
//   C  consumers: gate_up stages -> h (global)
//   -- grid barrier 2 (consumers; the producer keeps streaming down weights meanwhile) --
//   D  consumers: GeGLU + Q8_0 of this CTA's down experts' pairs, then the down stages -> y
//   -- grid barrier 3 --
//   E  every CTA combines a slice of the outputs: out = sum_j w_j * y_j in slot order.
constexpr int kFusedMaxT = 8;
constexpr int kFusedMaxP = kFusedMaxT * kMaxTopK;
static_assert(kFusedMaxT == kFusedTokens, "host and device chunk sizes differ");
constexpr int kFSlots = 5;
constexpr uint32_t kGridWaitLimit = 1u << 24;   // x >= 32 ns sleeps: bounded well under a second

enum : int32_t { ERR_GRID_TIMEOUT = 8 };

// Grid barrier word (per device, zero at load). Every CTA adds 1 to it except CTA 0, which adds
// 2^31 - (G - 1): once all G CTAs have arrived the word has gained exactly 2^31, so its top bit has
// flipped and its low 31 bits are back where they were (zero). No reset step is needed, and
// consecutive barriers and launches reuse the word; a partial sum never flips the top bit. Launches
// of the fused kernel cannot overlap (each fills every SM), so one word serves all of them.
__device__ unsigned int g_bar_word;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread per CTA: arrive, then wait (bounded) until the top bit of the word differs from the
// value this CTA saw at its own arrival.
__device__ __forceinline__ bool grid_barrier_thread(unsigned nblocks) {
    const unsigned add = blockIdx.x == 0 ? 0x80000000u - (nblocks - 1u) : 1u;
    __threadfence();
    const unsigned old = atomicAdd(&g_bar_word, add);
    for (uint32_t i = 0; i < kGridWaitLimit; ++i) {
        if ((ld_acquire_u32(&g_bar_word) ^ old) & 0x80000000u) {
            __threadfence();
            return true;
        }
        if (i >= 64) __nanosleep(32);
    }
    atomicOr(&g_error, ERR_GRID_TIMEOUT);
    return false;
}

struct FusedParams {
    const float *w_router, *b_router, *x;
    int32_t T, E, d, k, nff;
    NormArgs nrm;   // Gemma-4 block norms (nrm.pre == nullptr: none)
    double *nsum;   // [T][ceil(d / 64)] sums of squares of the combined output blocks (norms only)
    Residency res;
    PoolView hot_gu, cold_gu, hot_dn, cold_dn;
    float *logits;
    uint8_t *xq;
    int32_t xq_stride;
    float *h, *y, *out;
    int32_t *ids_out, *cnt_out, *off_out, *perm_out;
    float *w_out;
    uint8_t *qa;   // down activations (Q8_0 rows of n_ff) in expert-sorted slot order
    // completion counters, zeroed in phase A: gate_up rows done per (unique expert, 32-row ff block)
    // [kFusedMaxP][n_ff / 32], finished ff blocks per unique expert [kFusedMaxP], down rows done per
    // (token, 64-row block) [T][ceil(d / 64)], then combined output blocks per token [T]
    uint32_t *sync;
};

struct FusedRoute {
    int32_t ids[kFusedMaxP];
    float w[kFusedMaxP];
    int32_t cnt[kMaxE];
    int32_t off[kMaxE + 1];
    int32_t perm[kFusedMaxP];
    int32_t ecls[kMaxE], ewidx[kMaxE];   // residency class / pool index of every expert
    int32_t n_unique;
    int32_t uexp[kFusedMaxP], ucls[kFusedMaxP], uwidx[kFusedMaxP];
    uint32_t upre_gu[kFusedMaxP + 1], upre_dn[kFusedMaxP + 1];   // cumulative work units (see fused_dispatch)
    int32_t scan_c[kMaxE / 32], scan_u[kMaxE / 32];
    uint32_t scan_g[kMaxE / 32], scan_d[kMaxE / 32];
    int32_t split[4];   // this CTA's gate_up groups [g0, g1) and down groups [h0, h1)
    int32_t claim_gu, claim_dn;      // next unclaimed gate_up / down stage of this CTA
    int32_t claim[kGroups][2];       // each group's current claim (double-buffered by iteration)
    float red[kFusedMaxT][kConsumerWarps + 1];
    double dred[kFusedMaxT][kConsumerWarps + 1];
    float nscale[kFusedMaxT];        // rms_norm row scales of the tokens (Gemma-4 block norms)
    int32_t fin_n, fin[kFusedMaxT];  // tokens whose last output block this CTA combined (output norm)
};

struct FusedSmem {
    int route, bars, grid, xact, dact, slots, slot_cap, total;
};
__host__ __device__ inline FusedSmem fused_layout(int d, int nff) {
    FusedSmem L;
    int o = 0;
    L.route = o; o += (int)((sizeof(FusedRoute) + 127) / 128 * 128);
    L.bars = o;  o += ((2 * kFSlots + 1) * 8 + 127) / 128 * 128;
    L.grid = o;  o += MOE_IQ2S_GRID_ROWS * 8;
    L.xact = o;  o += kFusedMaxT * xq_stride_bytes(d);
    L.dact = o;  o += 2 * kFusedMaxT * q80_stride(nff);
    o = (o + 127) / 128 * 128;
    L.slots = o;
    const int gu = kGuStageRows * (int)row_bytes(T_Q4_K, d), dn = kDnStageRows * (int)row_bytes(T_Q5_0, nff);
    L.slot_cap = ((gu > dn ? gu : dn) + 16 + 127) / 128 * 128;
    o += kFSlots * L.slot_cap;
    L.total = o;
    return L;
}

// Order key of a routing candidate: the float's bits mapped to an unsigned order (-0 folded into +0,
// which compares equal to it), so the top-k's (value desc, index asc) becomes max key, then min index.
__device__ __forceinline__ uint32_t route_key(float v) {
    const uint32_t b = __float_as_uint(__fadd_rn(v, 0.f));
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Routing of the fused kernel, one warp per token (llama-graph.cpp:1553-1648): softmax max and sum
// over the token's logits, then k selection rounds (each a warp max over the lanes' best keys and a
// warp min over the tied experts' ids, so ties go to the lowest id), then the selected
// probabilities normalised by their slot-order sum.
__device__ void fused_route(const FusedParams &p, FusedRoute &rs, int tid) {
    const int T = p.T, E = p.E, k = p.k, lane = tid & 31, warp = tid >> 5, per = E / 32;
    for (int t = warp; t < T; t += kGemvThreads / 32) {
        float v[kMaxE / 32];
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) v[i] = i < per ? __ldcg(p.logits + (size_t)t * E + lane + 32 * i) : -INFINITY;
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) mx = fmaxf(mx, v[i]);
        mx = warp_max(mx);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) if (i < per) sum += expf(v[i] - mx);
        sum = warp_sum(sum);
        const float inv = 1.f / sum;
        uint32_t key[kMaxE / 32];
#pragma unroll
        for (int i = 0; i < kMaxE / 32; ++i) key[i] = i < per ? route_key(v[i]) : 0u;
        int my_id = 0;
        float my_v = 0.f;
        for (int j = 0; j < k; ++j) {
            uint32_t bk = 0u;
            int bi = 0;
#pragma unroll
            for (int i = 0; i < kMaxE / 32; ++i)
                if (key[i] > bk) { bk = key[i]; bi = i; }   // strict: the lowest i (lowest id) of a lane's ties
            const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
            const uint32_t e = __reduce_min_sync(0xffffffffu, bk == kmax ? (uint32_t)(lane + 32 * bi) : 0xffffffffu);
            if ((int)(e & 31) == lane) {
#pragma unroll
                for (int i = 0; i < kMaxE / 32; ++i)
                    if (i == (int)(e >> 5)) key[i] = 0u;   // taken (every real key is above 0)
            }
            const float ve = __shfl_sync(0xffffffffu, v[0], (int)(e & 31));
            float vs = ve;
#pragma unroll
            for (int i = 1; i < kMaxE / 32; ++i) {
                const float vi = __shfl_sync(0xffffffffu, v[i], (int)(e & 31));
                if (i == (int)(e >> 5)) vs = vi;
            }
            if (lane == j) { my_id = (int)e; my_v = vs; }
        }
        // probabilities of the selected experts, normalised by max(sum, 6.1e-5) with the sum taken in
        // slot order (llama-graph.cpp:1640-1648)
        const float pj = lane < k ? __fmul_rn(expf(my_v - mx), inv) : 0.f;
        float psum = 0.f;
        for (int j = 0; j < k; ++j) psum = __fadd_rn(psum, __shfl_sync(0xffffffffu, pj, j));
        psum = fmaxf(psum, 6.103515625e-5f);
        if (lane < k) {
            rs.ids[t * k + lane] = my_id;
            rs.w[t * k + lane] = __fdiv_rn(pj, psum);
        }
    }
    __syncthreads();
}

// work of an expert with n routed tokens for the split, in units that weigh the HBM bytes a CTA
// streams against the instructions its consumer warps issue (about 3 instructions per byte per SM at
// the measured bandwidth), rounded to a multiple of the expert's 8-row groups
__device__ __forceinline__ uint32_t fused_cost(const FusedParams &p, bool gu, int type, int n) {
    uint32_t bytes, instr;
    if (gu) {
        const uint32_t dec = type == T_Q4_K ? 24u : 70u;
        bytes = 8u * (uint32_t)row_bytes(type, p.d);
        instr = 8u * 8u * (uint32_t)(p.d / QK_K) * (dec + 16u * (uint32_t)n);
    } else {
        const uint32_t dec = type == T_IQ4_NL ? 45u : 25u;
        bytes = 8u * (uint32_t)(p.nff / QK32) * (type == T_IQ4_NL ? (uint32_t)B_IQ4_NL : (uint32_t)B_Q5_0);
        instr = 8u * (uint32_t)(p.nff / QK32) * (dec + 12u * (uint32_t)n);
    }
    const int gpe = gu ? 2 * p.nff / kGroupRows : p.d / kGroupRows;
    return (3u * bytes + instr) / 64u * (uint32_t)gpe;
}

// Histogram, exclusive scan and stable permutation of the routed pairs (ggml-cpu.c:1613-1626), and
// the unique-expert list with both projections' cumulative work units. Thread e owns expert e; the
// scan runs as E/32 warp shuffle scans plus the preceding warps' totals.
__device__ void fused_dispatch(const FusedParams &p, FusedRoute &rs, int tid, int nthreads) {
    const int P = p.T * p.k, E = p.E, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += nthreads) rs.cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < P; i += nthreads) {
        int e = rs.ids[i];
        if (e < 0 || e >= E) { atomicOr(&g_error, ERR_BAD_EXPERT); e = 0; rs.ids[i] = 0; }
        atomicAdd(&rs.cnt[e], 1);
    }
    __syncthreads();
    int c = 0, has = 0;
    uint32_t gc = 0, dc = 0;
    if (tid < E) {
        c = rs.cnt[tid];
        if (c > 0 && rs.ecls[tid] < 0) atomicOr(&g_error, ERR_BAD_EXPERT);   // its class pool is absent
        if (c > 0 && rs.ecls[tid] >= 0) {
            const bool hot = rs.ecls[tid] == 0;
            has = 1;
            gc = fused_cost(p, true, hot ? p.hot_gu.type : p.cold_gu.type, c);
            dc = fused_cost(p, false, hot ? p.hot_dn.type : p.cold_dn.type, c);
        }
    }
    int ci = c, ui = has;
    uint32_t gi = gc, di = dc;
    if (warp < E / 32) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a0 = __shfl_up_sync(0xffffffffu, ci, o), a1 = __shfl_up_sync(0xffffffffu, ui, o);
            const uint32_t a2 = __shfl_up_sync(0xffffffffu, gi, o), a3 = __shfl_up_sync(0xffffffffu, di, o);
            if (lane >= o) { ci += a0; ui += a1; gi += a2; di += a3; }
        }
        if (lane == 31) {
            rs.scan_c[warp] = ci;
            rs.scan_u[warp] = ui;
            rs.scan_g[warp] = gi;
            rs.scan_d[warp] = di;
        }
    }
    __syncthreads();
    if (tid < E) {
        for (int w = 0; w < warp; ++w) {
            ci += rs.scan_c[w];
            ui += rs.scan_u[w];
            gi += rs.scan_g[w];
            di += rs.scan_d[w];
        }
        rs.off[tid] = ci - c;
        if (has) {
            const int u = ui - 1;
            rs.uexp[u] = tid;
            rs.ucls[u] = rs.ecls[tid];
            rs.uwidx[u] = rs.ewidx[tid];
            rs.upre_gu[u + 1] = gi;
            rs.upre_dn[u + 1] = di;
        }
        if (tid == E - 1) {
            rs.off[E] = ci;
            rs.n_unique = ui;
            rs.upre_gu[0] = 0;
            rs.upre_dn[0] = 0;
        }
    }
    __syncthreads();
    for (int i = tid; i < P; i += nthreads) {
        const int e = rs.ids[i];
        int rank = 0;
        for (int q = 0; q < i; ++q) rank += rs.ids[q] == e;
        rs.perm[rs.off[e] + rank] = i;
    }
    __syncthreads();
}

// The 8-row group at position `pos` of a cumulative work prefix (every unique expert has gpe groups
// of equal cost), one warp: the unit u with pre[u] <= pos < pre[u + 1] by ballot, 32 units per step.
__device__ __forceinline__ int group_at_pre_warp(const uint32_t *pre, int U, uint32_t pos, int gpe, int lane) {
    if (pos >= pre[U]) return U * gpe;
    int u = 0;
    for (int u0 = 0; u0 < U; u0 += 32) {
        const int q = u0 + lane;
        const unsigned hit = __ballot_sync(0xffffffffu, q < U && pre[q] <= pos && pos < pre[q + 1]);
        if (hit) {
            u = u0 + __ffs(hit) - 1;
            break;
        }
    }
    const uint32_t unit = (pre[u + 1] - pre[u]) / (uint32_t)gpe;
    return u * gpe + (int)((pos - pre[u]) / unit);
}

// NRM: with the Gemma-4 block norms (p.nrm); a separate instance, so the plain layer's code is the
// same as without them
template <bool NRM>
__global__ void __launch_bounds__(kGemvThreads, 1) fused_decode_kernel(FusedParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, T = p.T, k = p.k, E = p.E, d = p.d, nff = p.nff, P = T * k;
    const FusedSmem L = fused_layout(d, nff);
    FusedRoute &rs = *reinterpret_cast<FusedRoute *>(smem + L.route);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *empty = full + kFSlots;
    uint64_t *xbar = empty + kFSlots;   // the Q8_K activation rows landed in xact
    uint64_t *grid = reinterpret_cast<uint64_t *>(smem + L.grid);
    uint8_t *xact = smem + L.xact;
    uint8_t *dact = smem + L.dact;
    uint8_t *slots = smem + L.slots;

    // ================= phase A
    if (warp == 0) FTRACE(0);
    const int nrb = (d + 63) / 64;
    if (blockIdx.x == 0)
        for (int i = tid; i < fused_sync_words(T, d, nff); i += kGemvThreads) p.sync[i] = 0u;
    {
        // the GELU table (128 KB) into L2 ahead of the GeGLU step: CTA b takes lines b, b + G, ...
        const char *gt = reinterpret_cast<const char *>(g_gelu_f16);
        for (int l = blockIdx.x + G * tid; l < (int)(sizeof(g_gelu_f16) / 128); l += G * kGemvThreads)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(gt + 128 * (size_t)l));
    }
    if (tid == 0) {
        for (int s = 0; s < kFSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarpsPerGroup);
        }
        mbar_init(xbar, 1);
        fence_mbar_init();
    }
    if (warp == kConsumerWarps) {
        // the producer warp is idle until phase B: residency classes and the IQ2_S codebook.
        // Loads are batched into registers before any shared-memory store, so they overlap.
        constexpr int kPer = kMaxE / 32;
        int slot[kPer], st[kPer], se[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = lane + 32 * i;
            slot[i] = (e < E && p.res.n_slots > 0 && p.res.exp_slot) ? __ldg(p.res.exp_slot + e) : -1;
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const bool in = slot[i] >= 0 && slot[i] < p.res.n_slots;
            st[i] = in ? __ldg(p.res.slot_state + slot[i]) : 0;
            se[i] = in ? __ldg(p.res.slot_exp + slot[i]) : -1;
        }
        uint64_t g[MOE_IQ2S_GRID_ROWS / 32];
#pragma unroll
        for (int i = 0; i < MOE_IQ2S_GRID_ROWS / 32; ++i) g[i] = g_iq2s_grid[lane + 32 * i];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = lane + 32 * i;
            if (e >= E) continue;
            // residency class of expert e (moert/cuda/ffn_moe.cu:101-104): 0 hot (slot), 1 cold, -1 no pool
            int cls = 1, widx = e;
            if (slot[i] >= 0 && slot[i] < p.res.n_slots && st[i] == 2 && se[i] == e) { cls = 0; widx = slot[i]; }
            const PoolView &pv = cls == 0 ? p.hot_gu : p.cold_gu;
            const PoolView &pd = cls == 0 ? p.hot_dn : p.cold_dn;
            if (pv.w == nullptr || pd.w == nullptr || widx >= pv.n) cls = -1;
            rs.ecls[e] = cls;
            rs.ewidx[e] = widx;
        }
#pragma unroll
        for (int i = 0; i < MOE_IQ2S_GRID_ROWS / 32; ++i) grid[lane + 32 * i] = g[i];
    }
    constexpr bool nrm = NRM;
    for (int unit = blockIdx.x; unit < E + T; unit += G) {
        if (unit < E) {
            // logits[t][unit] = W[unit] . x[t] (+ bias): every thread a strided share, then warp and
            // CTA reductions in a fixed order. With the Gemma-4 block norms the router input is
            // rms_norm(x[t]) / sqrt(d) * router_scale; its row scale s_t is factored out of the dot
            // (logit = s_t * (W . ((x / sqrt(d)) * router_scale)), equal to the dot of the per-value
            // rounded input to f32 rounding, like the summation order) and s_t comes from the
            // squares of the same x loads, so the logits need no pass over x ahead of them.
            const int n4 = d / 4;
            const float4 *w4 = reinterpret_cast<const float4 *>(p.w_router + (size_t)unit * d);
            const float4 *r4 = reinterpret_cast<const float4 *>(p.nrm.router);
            const float rc = nrm ? router_input_scale(d) : 1.f;
            float part[kFusedMaxT];
            double sq[kFusedMaxT];
#pragma unroll
            for (int t = 0; t < kFusedMaxT; ++t) {
                part[t] = 0.f;
                sq[t] = 0.0;
            }
            for (int i = tid; i < n4; i += kGemvThreads) {
                const float4 w = __ldg(w4 + i);
                const float4 r = nrm ? __ldg(r4 + i) : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
                for (int t = 0; t < kFusedMaxT; ++t) {
                    if (t < T) {
                        float4 xv = __ldg(reinterpret_cast<const float4 *>(p.x + (size_t)t * d) + i);
                        if (nrm) {
                            sq[t] += sq_sum4(xv);
                            xv = router_input4(xv, 1.f, rc, r);
                        }
                        part[t] = fmaf(w.x, xv.x, part[t]);
                        part[t] = fmaf(w.y, xv.y, part[t]);
                        part[t] = fmaf(w.z, xv.z, part[t]);
                        part[t] = fmaf(w.w, xv.w, part[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < kFusedMaxT; ++t) {
                if (t < T) {
                    const float v = warp_sum(part[t]);
                    if (lane == 0) rs.red[t][warp] = v;
                }
            }
            if (nrm) {   // all tokens' squares reduced together (absent tokens reduce zeros)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                    for (int t = 0; t < kFusedMaxT; ++t) sq[t] += __shfl_xor_sync(0xffffffffu, sq[t], o);
                }
                if (lane == 0) {
#pragma unroll
                    for (int t = 0; t < kFusedMaxT; ++t)
                        if (t < T) rs.dred[t][warp] = sq[t];
                }
            }
            __syncthreads();
            if (tid < T) {
                float v = 0.f;
                for (int w = 0; w < kConsumerWarps + 1; ++w) v += rs.red[tid][w];
                if (nrm) {
                    double q = 0.0;
                    for (int w = 0; w < kConsumerWarps + 1; ++w) q += rs.dred[tid][w];
                    v = __fmul_rn(v, rms_row_scale(q, d, p.nrm.eps));
                }
                if (p.b_router) v = __fadd_rn(v, p.b_router[unit]);
                p.logits[(size_t)tid * E + unit] = v;
            }
            __syncthreads();
        } else if (nrm) {
            // token t's Q8_K row of the expert input rms_norm(x[t]) * pre_norm: one warp per
            // super-block (d <= 4096 for the block norms), the row scale from the warps' squares
            const int t = unit - E, nsb = d / QK_K;
            uint8_t *row = p.xq + (size_t)t * p.xq_stride;
            float4 xa = make_float4(0.f, 0.f, 0.f, 0.f), xb = xa;
            if (warp < nsb) {
                const float4 *x4 = reinterpret_cast<const float4 *>(p.x + (size_t)t * d + warp * QK_K);
                xa = __ldg(x4 + 2 * lane);
                xb = __ldg(x4 + 2 * lane + 1);
            }
            const double q = warp_sum_d(sq_sum4(xa) + sq_sum4(xb));
            if (lane == 0) rs.dred[0][warp] = q;
            __syncthreads();
            if (tid == 0) {
                double tot = 0.0;
                for (int w = 0; w < nsb; ++w) tot += rs.dred[0][w];
                rs.nscale[0] = rms_row_scale(tot, d, p.nrm.eps);
            }
            __syncthreads();
            if (warp < nsb) {
                const float sc = rs.nscale[0];
                const float4 *pw = reinterpret_cast<const float4 *>(p.nrm.pre + warp * QK_K);
                const float4 na = norm_weight4(xa, sc, __ldg(pw + 2 * lane)), nb = norm_weight4(xb, sc, __ldg(pw + 2 * lane + 1));
                float v[8] = {na.x, na.y, na.z, na.w, nb.x, nb.y, nb.z, nb.w};
                q8k_quantize_warp(v, reinterpret_cast<int8_t *>(row) + warp * 256,
                                  reinterpret_cast<float *>(row + nsb * 256) + warp,
                                  reinterpret_cast<int16_t *>(row + nsb * 256 + nsb * 4) + warp * 16, lane);
            }
            __syncthreads();
        } else {
            const int t = unit - E, nsb = d / QK_K;
            uint8_t *row = p.xq + (size_t)t * p.xq_stride;
            for (int sb = warp; sb < nsb; sb += kGemvThreads / 32)
                q8k_superblock_warp(p.x + (size_t)t * d + sb * 256, reinterpret_cast<int8_t *>(row) + sb * 256,
                                    reinterpret_cast<float *>(row + nsb * 256) + sb,
                                    reinterpret_cast<int16_t *>(row + nsb * 256 + nsb * 4) + sb * 16, lane);
        }
    }
    __syncthreads();
    if (warp == 0) FTRACE(1);
    if (tid == 0) grid_barrier_thread(G);
    __syncthreads();
    if (tid == kConsumerWarps * 32) {
        // every token's Q8_K row (written by other CTAs before the barrier) into xact, in the
        // background of the routing; the generic-proxy writes are ordered before this async-proxy read
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_expect_tx(xbar, (uint32_t)(T * p.xq_stride));
        bulk_g2s(xact, p.xq, (uint32_t)(T * p.xq_stride), xbar);
    }
    if (warp == 0) FTRACE(2);

    // ================= phase B: routing and the work split
    fused_route(p, rs, tid);
    if (warp == 0) FTRACE(3);
    fused_dispatch(p, rs, tid, kGemvThreads);
    if (warp == 0) FTRACE(4);
#ifdef MOEB_TRACE
    fused_dispatch(p, rs, tid, kGemvThreads);   // second, warm pass (trace builds only)
    if (warp == 0) FTRACE(15);
#endif
    if (blockIdx.x == 0) {
        for (int i = tid; i < P; i += kGemvThreads) {
            if (p.ids_out) p.ids_out[i] = rs.ids[i];
            if (p.w_out) p.w_out[i] = rs.w[i];
            if (p.perm_out) p.perm_out[i] = rs.perm[i];
        }
        for (int e = tid; e <= E; e += kGemvThreads) {
            if (p.cnt_out && e < E) p.cnt_out[e] = rs.cnt[e];
            if (p.off_out) p.off_out[e] = rs.off[e];
        }
    }
    if (warp == 0) FTRACE(13);
    const int U = rs.n_unique;
    const int gpe_gu = 2 * nff / kGroupRows, sg_gu = kGuStageRows / kGroupRows, spe_gu = (gpe_gu + sg_gu - 1) / sg_gu;
    const int gpe_dn = d / kGroupRows, sg_dn = kDnStageRows / kGroupRows, spe_dn = (gpe_dn + sg_dn - 1) / sg_dn;
    // work-balanced share of each projection (totals stay below 2^32 / G units): warps 0-3 search
    // the bounds g0, g1 (gate_up) and h0, h1 (down) at once
    if (warp < 4) {
        const bool gu = warp < 2;
        const uint32_t *pre = gu ? rs.upre_gu : rs.upre_dn;
        const uint32_t pos = pre[U] * (blockIdx.x + (uint32_t)(warp & 1)) / (uint32_t)G;
        const int g = group_at_pre_warp(pre, U, pos, gu ? gpe_gu : gpe_dn, lane);
        if (lane == 0) rs.split[warp] = g;
    }
    if (tid == 0) {
        rs.claim_gu = 0;
        rs.claim_dn = 0;
    }
    __syncthreads();
    const int g0 = rs.split[0], g1 = rs.split[1], h0 = rs.split[2], h1 = rs.split[3];
    if (warp == 0) FTRACE(14);
    const int Sg = g1 > g0 ? stage_of(g0, gpe_gu, spe_gu, sg_gu) : 0;
    const int n_gu = g1 > g0 ? stage_of(g1 - 1, gpe_gu, spe_gu, sg_gu) - Sg + 1 : 0;
    const int Sd = h1 > h0 ? stage_of(h0, gpe_dn, spe_dn, sg_dn) : 0;
    const int n_dn = h1 > h0 ? stage_of(h1 - 1, gpe_dn, spe_dn, sg_dn) - Sd + 1 : 0;
    if (warp == 0) FTRACE(12);

    auto plan = [&](int it, bool &is_gu) -> StagePlan {
        is_gu = it < n_gu;
        return is_gu ? stage_plan(Sg + it, g0, g1, gpe_gu, spe_gu, sg_gu)
                     : stage_plan(Sd + (it - n_gu), h0, h1, gpe_dn, spe_dn, sg_dn);
    };

    if (warp == kConsumerWarps) {
        // ================= producer: gate_up stages, then down stages, through one slot ring
        if (lane == 0) {
            for (int it = 0; it < n_gu + n_dn; ++it) {
                const int slot = it % kFSlots;
                if (it >= kFSlots && !mbar_wait(&empty[slot], (uint32_t)(((it / kFSlots) - 1) & 1))) break;
                bool is_gu;
                const StagePlan st = plan(it, is_gu);
                const bool hot = rs.ucls[st.u] == 0;
                const PoolView &pv = is_gu ? (hot ? p.hot_gu : p.cold_gu) : (hot ? p.hot_dn : p.cold_dn);
                const int d_in = is_gu ? d : nff, d_out = is_gu ? 2 * nff : d;
                const int rb = (int)row_bytes(pv.type, d_in);
                const uint32_t bytes = (uint32_t)(st.nrows * rb);
                mbar_expect_tx(&full[slot], bytes);
                bulk_g2s(slots + slot * L.slot_cap, pool_entry(pv, rs.uwidx[st.u], d_out, d_in) + (size_t)st.row0 * rb,
                         bytes, &full[slot]);
            }
        }
    } else {
        // ================= consumers
        const int nsb = d / QK_K, nb = nff / QK32;
        const int xs = p.xq_stride, as = q80_stride(nff);
        const size_t hpart = (size_t)T * k * 2 * nff;   // stride of the four gate_up partial-sum parts
        const int qas = fused_qa_stride(nff);
        uint32_t *blk_cnt = p.sync, *act_cnt = p.sync + kFusedMaxP * nb, *dn_cnt = act_cnt + kFusedMaxP;
        uint32_t *tok_cnt = dn_cnt + T * nrb;
        const int grp = warp / kWarpsPerGroup, wg = warp % kWarpsPerGroup;
        uint32_t kv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            kv[i] = (uint32_t)(uint8_t)g_iq4nl[4 * i] | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 1] << 8) |
                    ((uint32_t)(uint8_t)g_iq4nl[4 * i + 2] << 16) | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 3] << 24);
        bool ok = mbar_wait(xbar, 0u);
        if (warp == 0) FTRACE(5);
        // ---- phase C: gate_up. Groups claim stages in order as they become free (lane 0 of the
        // group's first warp takes the next index; the group reads it after a group barrier).
        for (int m = 0;; ++m) {
            if (wg == 0 && lane == 0) rs.claim[grp][m & 1] = atomicAdd(&rs.claim_gu, 1);
            group_sync(grp);
            const int it = rs.claim[grp][m & 1];
            if (it >= n_gu) break;
            const int slot = it % kFSlots;
            STRACE(it, 0);
            if (ok && !mbar_wait(&full[slot], (uint32_t)((it / kFSlots) & 1))) ok = false;
            STRACE(it, 1);
            bool is_gu;
            const StagePlan st = plan(it, is_gu);
            const int e = rs.uexp[st.u];
            const bool hot = rs.ucls[st.u] == 0;
            const int type = hot ? p.hot_gu.type : p.cold_gu.type;
            const int rb = (int)row_bytes(type, d);
            const int po = rs.off[e], n = rs.cnt[e];
            const int j = lane & 7, r = wg * 4 + (lane >> 3);
            if (ok && wg * 4 < st.nrows) {
                const uint8_t *row = slots + slot * L.slot_cap + (size_t)r * rb;
                for (int c0 = 0; c0 < n; c0 += kTokChunk) {
                    const int nt = min(kTokChunk, n - c0);
                    int tok[kTokChunk], pair[kTokChunk];
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        pair[c] = rs.perm[po + c0 + (c < nt ? c : 0)];
                        tok[c] = pair[c] / k;
                    }
                    float v[4] = {0.f, 0.f, 0.f, 0.f};
                    // one- and four-column bodies only (short code); missing columns repeat column 0
                    if (nt == 1) gu_rows<1>(row, nsb, j, type, grid, xact, xs, tok, v);
                    else gu_rows<4>(row, nsb, j, type, grid, xact, xs, tok, v);
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        if (j == 0 && c < nt) {
                            float *hp = p.h + (size_t)pair[c] * 2 * nff + st.row0 + r;
                            hp[0] = v[c];
                            hp[hpart] = 0.f;   // rows not split over the four parts
                            hp[2 * hpart] = 0.f;
                            hp[3 * hpart] = 0.f;
                        }
                    }
                }
            }
            __syncwarp();
            STRACE(it, 2);
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        consumer_sync();
        if (warp == 0) FTRACE(6);
        // ---- phase D1: publish this CTA's gate_up rows per (expert, 32-row ff block), one count per
        // 8-row group; the CTA whose count completes a block's 64 rows (32 gate + 32 up) computes that
        // block's GeGLU + Q8_0 for every token of the expert into qa, then counts the block as done.
        // Each counting thread fences first, which orders the whole CTA's h rows (made visible to it by
        // the barrier above) before its count.
        int *blk_todo = reinterpret_cast<int *>(dact);   // act items: (u * nb + b) * kFusedMaxT + token
        const int todo_cap = 2 * kFusedMaxT * as / 4 - 1;
        if (tid == 0) blk_todo[0] = 0;
        consumer_sync();
        for (int gg = g0 + tid; gg < g1; gg += kConsumerWarps * 32) {
            const int u = gg / gpe_gu, r = (gg - u * gpe_gu) * kGroupRows;
            const int b = (r < nff ? r : r - nff) / QK32;
            __threadfence();
            if (atomicAdd(&blk_cnt[u * nb + b], (uint32_t)kGroupRows) + kGroupRows == 2u * QK32) {
                const int n = min(rs.cnt[rs.uexp[u]], T);
                const int at = atomicAdd(&blk_todo[0], n);
                if (at + n <= todo_cap) {
                    for (int i = 0; i < n; ++i) blk_todo[1 + at + i] = (u * nb + b) * kFusedMaxT + i;
                } else {
                    atomicOr(&g_error, ERR_CAPACITY);
                }
            }
        }
        consumer_sync();
        const int n_items = min(blk_todo[0], todo_cap);
        if (n_items > 0) {
            if (tid == 0) __threadfence();   // every other CTA's rows of these blocks are counted
            consumer_sync();
            // two items per warp in flight: both items' partial sums are loaded before either is quantised
            for (int q0 = warp; q0 < n_items; q0 += 2 * kConsumerWarps) {
                float g[2], v[2];
                uint8_t *row[2];
                int bq[2];
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    const int q = q0 + h2 * kConsumerWarps;
                    g[h2] = v[h2] = 0.f;
                    row[h2] = nullptr;
                    bq[h2] = 0;
                    if (q < n_items) {
                        const int item = blk_todo[1 + q], ub = item / kFusedMaxT, i = item - ub * kFusedMaxT;
                        const int u = ub / nb, b = ub - u * nb, e = rs.uexp[u];
                        const float *hp = p.h + (size_t)rs.perm[rs.off[e] + i] * 2 * nff + QK32 * b + lane;
                        // gate_up partial sums of the four super-block quarters, added in order
                        g[h2] = __fadd_rn(__fadd_rn(__fadd_rn(__ldcg(hp), __ldcg(hp + hpart)), __ldcg(hp + 2 * hpart)),
                                          __ldcg(hp + 3 * hpart));
                        v[h2] = __fadd_rn(__fadd_rn(__fadd_rn(__ldcg(hp + nff), __ldcg(hp + nff + hpart)),
                                                    __ldcg(hp + nff + 2 * hpart)),
                                          __ldcg(hp + nff + 3 * hpart));
                        row[h2] = p.qa + (size_t)(rs.off[e] + i) * qas;
                        bq[h2] = b;
                    }
                }
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    if (row[h2] == nullptr) continue;
                    const int b = bq[h2];
                    q80_block_warp(geglu1(g[h2], v[h2]), reinterpret_cast<int8_t *>(row[h2]) + QK32 * b,
                                   reinterpret_cast<float *>(row[h2] + nb * 32) + b,
                                   reinterpret_cast<int *>(row[h2] + nb * 36) + b, lane);
                }
            }
            consumer_sync();
            for (int q = tid; q < n_items; q += kConsumerWarps * 32) {
                const int item = blk_todo[1 + q];
                if (item % kFusedMaxT == 0) {   // one count per finished block
                    __threadfence();
                    atomicAdd(&act_cnt[item / kFusedMaxT / nb], 1u);
                }
            }
        }

        // ---- phase D2: the down activations of this CTA's down experts (<= 2) once all their
        // blocks are finished (bounded wait), copied into shared memory
        const int u_first = h1 > h0 ? h0 / gpe_dn : 0;
        const int u_last = h1 > h0 ? (h1 - 1) / gpe_dn : -1;
        if (u_last - u_first > 1 && tid == 0) atomicOr(&g_error, ERR_CAPACITY);
        if (tid == 0) {
            for (int u = u_first; u <= min(u_last, u_first + 1); ++u) {
                uint32_t i = 0;
                while (ld_acquire_u32(&act_cnt[u]) < (uint32_t)nb) {
                    if (++i >= kGridWaitLimit) { atomicOr(&g_error, ERR_GRID_TIMEOUT); break; }
                    if (i >= 64) __nanosleep(32);
                }
            }
            __threadfence();
        }
        consumer_sync();
        if (warp == 0) FTRACE(7);
        for (int u = u_first; u <= min(u_last, u_first + 1); ++u) {
            const int e = rs.uexp[u], n = min(rs.cnt[e], T), r16 = as / 16;
            for (int i = tid; i < n * r16; i += kConsumerWarps * 32) {
                const int row = i / r16, c = i - row * r16;
                reinterpret_cast<int4 *>(dact + (size_t)((u - u_first) * T + row) * as)[c] =
                    __ldcg(reinterpret_cast<const int4 *>(p.qa + (size_t)(rs.off[e] + row) * qas) + c);
            }
        }
        consumer_sync();
        if (warp == 0) FTRACE(8);
        // the unified sequence continues at it = n_gu; groups keep their residue
        for (int m = 0;; ++m) {
            if (wg == 0 && lane == 0) rs.claim[grp][m & 1] = n_gu + atomicAdd(&rs.claim_dn, 1);
            group_sync(grp);
            const int it = rs.claim[grp][m & 1];
            if (it >= n_gu + n_dn) break;
            const int slot = it % kFSlots;
            STRACE(it, 0);
            if (ok && !mbar_wait(&full[slot], (uint32_t)((it / kFSlots) & 1))) ok = false;
            STRACE(it, 1);
            bool is_gu;
            const StagePlan st = plan(it, is_gu);
            const int e = rs.uexp[st.u], widx = rs.uwidx[st.u];
            const bool hot = rs.ucls[st.u] == 0;
            const PoolView &pv = hot ? p.hot_dn : p.cold_dn;
            const int rb = (int)row_bytes(pv.type, nff);
            const int po = rs.off[e];
            int n = rs.cnt[e];
            if (n > T) {
                if (lane == 0) atomicOr(&g_error, ERR_CAPACITY);
                n = T;
            }
            const int half = lane & 1, r = wg * 16 + (lane >> 1);
            const int bmid = (nb + 1) / 2, b0 = half ? bmid : 0, b1 = half ? nb : bmid;
            const bool valid = r < st.nrows;
            const int slot0 = (st.u - u_first) * T;
            if (ok && wg * 16 < st.nrows) {
                const uint8_t *row = slots + slot * L.slot_cap + (size_t)(valid ? r : 0) * rb;
                for (int c0 = 0; c0 < n; c0 += kTokChunk) {
                    const int nt = min(kTokChunk, n - c0);
                    float v[4] = {0.f, 0.f, 0.f, 0.f};
                    if (nt == 1) dn_rows<1>(row, b0, b1, nb, pv.type, kv, dact, as, slot0 + c0, nt, v);
                    else dn_rows<4>(row, b0, b1, nb, pv.type, kv, dact, as, slot0 + c0, nt, v);
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        float sum = v[c];
                        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                        if (half == 0 && valid && c < nt) {
                            const int pair = rs.perm[po + c0 + c];
                            if (pv.scale) sum = __fmul_rn(sum, pv.scale[widx]);
                            p.y[(size_t)pair * d + st.row0 + r] = sum;
                        }
                    }
                }
            }
            __syncwarp();
            STRACE(it, 2);
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (warp == 0) FTRACE(10);
        // ---- phase E: publish this CTA's down rows per (token, 64-row block); the CTA whose
        // count completes a block combines it: out[t] = sum_j w_j * y[t*k + j], products rounded,
        // then added in slot order (ggml_mul + the view-add chain, llama-graph.cpp:1814-1848)
        consumer_sync();
        int *todo = reinterpret_cast<int *>(dact);   // the activations are no longer needed
        if (tid == 0) {
            todo[0] = 0;
            if (nrm) rs.fin_n = 0;
            __threadfence();
        }
        consumer_sync();
        if (h1 > h0) {
            // one (pair, block) item per thread, so the counting atomics travel together; each
            // counting thread fences first, which orders the whole CTA's y rows (made visible to it
            // by the barrier above) before its count
            __threadfence();
            int items = 0;
            for (int u = h0 / gpe_dn; u <= (h1 - 1) / gpe_dn; ++u) {
                const int lo = max(h0, u * gpe_dn) * kGroupRows - u * d, hi = min(h1, (u + 1) * gpe_dn) * kGroupRows - u * d;
                const int e = rs.uexp[u], po = rs.off[e], n = min(rs.cnt[e], T);
                const int rb0 = lo / 64, rb1 = (hi - 1) / 64;
                for (int c = 0; c < n; ++c)
                    for (int rb = rb0; rb <= rb1; ++rb, ++items) {
                        if (items % (kConsumerWarps * 32) != tid) continue;
                        const int rows = min(hi, (rb + 1) * 64) - max(lo, rb * 64);
                        const int t = rs.perm[po + c] / k;
                        const uint32_t before = atomicAdd(&dn_cnt[t * nrb + rb], (uint32_t)rows);
                        if (before + rows == (uint32_t)(k * min(64, d - rb * 64))) {
                            const int at = atomicAdd(&todo[0], 1);
                            todo[1 + 2 * at] = t;
                            todo[2 + 2 * at] = rb;
                        }
                    }
            }
        }
        consumer_sync();
        if (warp == 0) FTRACE(11);
        const int n_todo = todo[0];
        if (n_todo > 0) {
            if (tid == 0) __threadfence();
            consumer_sync();
            for (int q = warp; q < n_todo; q += kConsumerWarps) {
                const int t = todo[1 + 2 * q], rb = todo[2 + 2 * q];
                double sq = 0.0;
                for (int rr = lane; rr < min(64, d - rb * 64); rr += 32) {
                    const int row = rb * 64 + rr;
                    float acc = __fmul_rn(__ldcg(p.y + (size_t)(t * k) * d + row), rs.w[t * k]);
                    for (int j = 1; j < k; ++j)
                        acc = __fadd_rn(acc, __fmul_rn(__ldcg(p.y + (size_t)(t * k + j) * d + row), rs.w[t * k + j]));
                    p.out[(size_t)t * d + row] = acc;
                    if (nrm) sq += (double)__fmul_rn(acc, acc);
                }
                if (nrm) {
                    // the output norm (ffn_post_norm_2): the block's sum of squares, then a count
                    // per token; the CTA that combines the token's last block scales its row below
                    sq = warp_sum_d(sq);
                    if (lane == 0) p.nsum[t * nrb + rb] = sq;
                    asm volatile("fence.acq_rel.gpu;" ::: "memory");   // this lane's out rows (and sum) first
                    __syncwarp();
                    if (lane == 0 && atomicAdd(&tok_cnt[t], 1u) + 1u == (uint32_t)nrb) {
                        asm volatile("fence.acq_rel.gpu;" ::: "memory");
                        rs.fin[atomicAdd(&rs.fin_n, 1)] = t;
                    }
                }
            }
        }
        if (nrm) {
            consumer_sync();
            const int nf = rs.fin_n;
            if (nf > 0) {
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                const int n4 = d / 4, i0 = tid, i1 = tid + kConsumerWarps * 32;   // d <= 4096: two per thread
                const float4 *w4 = reinterpret_cast<const float4 *>(p.nrm.post);
                for (int f = 0; f < nf; ++f) {
                    const int t = rs.fin[f];
                    float4 *o4 = reinterpret_cast<float4 *>(p.out + (size_t)t * d);
                    // this thread's share of the row and the blocks' sums, loaded together; every warp
                    // sums the blocks lane-strided then by the xor tree (one fixed order, so all warps,
                    // in whichever CTA finishes the token, form the same scale)
                    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0, w0 = v0, w1 = v0;
                    if (i0 < n4) { v0 = __ldcg(o4 + i0); w0 = __ldg(w4 + i0); }
                    if (i1 < n4) { v1 = __ldcg(o4 + i1); w1 = __ldg(w4 + i1); }
                    double part = 0.0;
                    for (int b = lane; b < nrb; b += 32) part += __ldcg(p.nsum + t * nrb + b);
                    const float sc = rms_row_scale(warp_sum_d(part), d, p.nrm.eps);
                    if (i0 < n4) o4[i0] = norm_weight4(v0, sc, w0);
                    if (i1 < n4) o4[i1] = norm_weight4(v1, sc, w1);
                }
            }
        }
    }
    if (warp == 0) FTRACE(9);
}

}  // namespace moeb

#include "prefill.cuh"
#include "gateup_lx.cuh"
#include "mid.cuh"

namespace moeb {

// ------------------------------------------------------------------ Q8_K activations for the per-kind path
__global__ void __launch_bounds__(kThreads) quant_q8k_kernel(const float *x, uint8_t *dst, int d, int stride) {
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nsb = d / QK_K;
    uint8_t *row = dst + (size_t)t * stride;
    for (int sb = warp; sb < nsb; sb += kWarps)
        q8k_superblock_warp(x + (size_t)t * d + sb * 256, reinterpret_cast<int8_t *>(row) + sb * 256,
                            reinterpret_cast<float *>(row + nsb * 256) + sb,
                            reinterpret_cast<int16_t *>(row + nsb * 256 + nsb * 4) + sb * 16, lane);
}

// ------------------------------------------------------------------ standalone routing / dispatch
__global__ void __launch_bounds__(kThreads, 1) route_only_kernel(RouteSrc r, int32_t *ids, float *w, int32_t *cnt,
                                                                 int32_t *off, int32_t *perm) {
    __shared__ RouteSmem rs;
    const int tid = threadIdx.x;
    route_tokens(r, rs, tid, kThreads / 32);
    __syncthreads();
    const Residency none = {0, nullptr, nullptr, nullptr};
    const PoolView pv = {nullptr, T_Q4_K, 0, nullptr, nullptr};
    dispatch_pairs(r, none, pv, pv, QK_K, kGroupRows, rs, tid, kThreads, false);
    const int P = r.T * r.k;
    for (int i = tid; i < P; i += kThreads) {
        if (ids) ids[i] = rs.ids[i];
        if (w) w[i] = rs.w[i];
        if (perm) perm[i] = rs.perm[i];
    }
    for (int e = tid; e <= r.E; e += kThreads) {
        if (cnt && e < r.E) cnt[e] = rs.cnt[e];
        if (off) off[e] = rs.off[e];
    }
}

// ------------------------------------------------------------------ dequantisation (bit-exact)
// One thread per 32 output values. Products are rounded exactly as the ggml dequantisers write
// them (ggml-quants.c:442,1471,2416,2471,2653; Q8_0 as dequantize_row_q8_0): no fused multiply-add.
__global__ void dequant_kernel(int32_t type, const uint8_t *src, float *dst, int64_t rows, int64_t n) {
    const int64_t nchunk = n / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nchunk) return;
    const int64_t r = i / nchunk, c = i - r * nchunk;
    const uint8_t *row = src + r * row_bytes(type, n);
    float *y = dst + r * n + c * 32;
    if (type == T_Q4_K) {
        const uint8_t *blk = row + (c / 8) * B_Q4_K;
        const int j = (int)(c % 8);
        const float d = h2f(ld_u16(blk)), dmin = h2f(ld_u16(blk + 2));
        const uint8_t *sc = blk + 4;
        int s, m;
        if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
        else { s = (sc[j + 4] & 0x0f) | ((sc[j - 4] >> 6) << 4); m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4); }
        const float d1 = __fmul_rn(d, (float)s), m1 = __fmul_rn(dmin, (float)m);
        const uint8_t *q = blk + 16 + 32 * (j / 2);
        for (int l = 0; l < 32; ++l) {
            const int v = (j & 1) ? (q[l] >> 4) : (q[l] & 0xf);
            y[l] = __fsub_rn(__fmul_rn(d1, (float)v), m1);
        }
    } else if (type == T_IQ2_S) {
        const uint8_t *blk = row + (c / 8) * B_IQ2_S;
        const int ib = (int)(c % 8);
        const float d = h2f(ld_u16(blk));
        const uint8_t sc = blk[74 + ib];
        const float db0 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc & 0xf))), 0.25f);
        const float db1 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc >> 4))), 0.25f);
        for (int l = 0; l < 4; ++l) {
            const int g = 4 * ib + l;
            const int gi = blk[2 + g] | (((blk[66 + ib] >> (2 * l)) & 3) << 8);
            const uint64_t gv = g_iq2s_grid[gi];
            const uint8_t sg = blk[34 + g];
            const float dl = l < 2 ? db0 : db1;
            for (int jj = 0; jj < 8; ++jj) {
                const float mag = (float)((gv >> (8 * jj)) & 0xff);
                y[8 * l + jj] = __fmul_rn(__fmul_rn(dl, mag), ((sg >> jj) & 1) ? -1.f : 1.f);
            }
        }
    } else if (type == T_IQ2_XXS) {
        // 32-value group ib: four codebook rows, four sign patterns, one sub-scale
        const uint8_t *blk = row + (c / 8) * B_IQ2_XXS;
        const uint8_t *g8 = blk + 2 + 8 * (c % 8);
        const float d = h2f(ld_u16(blk));
        const uint32_t hi = (uint32_t)g8[4] | ((uint32_t)g8[5] << 8) | ((uint32_t)g8[6] << 16) | ((uint32_t)g8[7] << 24);
        const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(hi >> 28))), 0.25f);
        for (int l = 0; l < 4; ++l) {
            const uint64_t gv = g_iq2xxs_grid[g8[l]];
            const uint8_t sg = g_iq2xxs_signs[(hi >> (7 * l)) & 127];
            for (int jj = 0; jj < 8; ++jj)
                y[8 * l + jj] = __fmul_rn(__fmul_rn(db, (float)((gv >> (8 * jj)) & 0xff)), ((sg >> jj) & 1) ? -1.f : 1.f);
        }
    } else if (type == T_Q8_0) {
        const uint8_t *blk = row + c * B_Q8_0;
        const float d = h2f(ld_u16(blk));
        for (int jj = 0; jj < 32; ++jj) y[jj] = __fmul_rn((float)(int8_t)blk[2 + jj], d);
    } else if (type == T_Q5_0) {
        const uint8_t *blk = row + c * B_Q5_0;
        const float d = h2f(ld_u16(blk));
        const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
        for (int jj = 0; jj < 16; ++jj) {
            const int v0 = (int)((blk[6 + jj] & 0xf) | (((qh >> jj) & 1) << 4)) - 16;
            const int v1 = (int)((blk[6 + jj] >> 4) | (((qh >> (jj + 16)) & 1) << 4)) - 16;
            y[jj] = __fmul_rn((float)v0, d);
            y[jj + 16] = __fmul_rn((float)v1, d);
        }
    } else if (type == T_IQ4_NL) {
        const uint8_t *blk = row + c * B_IQ4_NL;
        const float d = h2f(ld_u16(blk));
        for (int jj = 0; jj < 16; ++jj) {
            y[jj] = __fmul_rn(d, (float)g_iq4nl[blk[2 + jj] & 0xf]);
            y[jj + 16] = __fmul_rn(d, (float)g_iq4nl[blk[2 + jj] >> 4]);
        }
    }
}

// Activation quantisation to ggml's own block layouts (block_q8_K / block_q8_0), for inspection.
__global__ void __launch_bounds__(kThreads) quant_act_kernel(int32_t vdt, const float *x, uint8_t *dst, int64_t n) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t r = blockIdx.x;
    const float *xr = x + r * n;
    uint8_t *out = dst + r * row_bytes(vdt, n);
    if (vdt == T_Q8_K) {
        for (int64_t sb = warp; sb < n / QK_K; sb += kWarps) {
            uint8_t *blk = out + sb * B_Q8_K;
            float d;
            int16_t bs[1];
            __shared__ int8_t qs[kWarps][256];
            __shared__ int16_t bsum[kWarps][16];
            q8k_superblock_warp(xr + sb * 256, qs[warp], &d, bsum[warp], lane);
            __syncwarp();
            (void)bs;
            for (int i = lane; i < 256; i += 32) blk[4 + i] = (uint8_t)qs[warp][i];
            if (lane < 16) { blk[260 + 2 * lane] = (uint8_t)(bsum[warp][lane] & 0xff); blk[261 + 2 * lane] = (uint8_t)((uint16_t)bsum[warp][lane] >> 8); }
            if (lane == 0) { uint32_t u = __float_as_uint(d); blk[0] = u & 0xff; blk[1] = (u >> 8) & 0xff; blk[2] = (u >> 16) & 0xff; blk[3] = u >> 24; }
            __syncwarp();
        }
    } else {
        for (int64_t b = warp; b < n / QK32; b += kWarps) {
            __shared__ int8_t qs[kWarps][32];
            __shared__ float dd[kWarps];
            __shared__ int qsum[kWarps];
            q80_block_warp(xr[b * 32 + lane], qs[warp], &dd[warp], &qsum[warp], lane);
            __syncwarp();
            uint8_t *blk = out + b * B_Q8_0;
            blk[2 + lane] = (uint8_t)qs[warp][lane];
            if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = f2h_rn(dd[warp]);   // blocks sit at even offsets
            __syncwarp();
        }
    }
}

// ------------------------------------------------------------------ host launchers
static cudaError_t launch_ex(const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             void **args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

size_t gemv_smem_bytes(int kind, int d_in, int T) { return (size_t)gemv_layout(kind == 0 ? 0 : 1, d_in, T).total; }

// Opt-in to more than 48 KB of dynamic shared memory, once per device and kernel.
static cudaError_t smem_optin(const void *fn, size_t bytes, unsigned *done_mask, int bit) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 32) return cudaErrorInvalidDevice;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (done_mask[dev] & (1u << bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done_mask[dev] |= 1u << bit;
    return e;
}

cudaError_t launch_gemv(const GemvParams &p, cudaStream_t s, bool pdl, int n_sms) {
    const size_t smem = gemv_smem_bytes(p.kind, p.d_in, p.route.T);
    static unsigned optin[32];
    const cudaError_t e = smem_optin((const void *)gemv_kernel, 227 * 1024, optin, 0);
    if (e != cudaSuccess) return e;
    GemvParams q = p;
    void *args[] = {&q};
    return launch_ex((const void *)gemv_kernel, dim3(n_sms), dim3(kGemvThreads), smem, s, pdl, args);
}

size_t fused_smem_bytes(int d, int nff) { return (size_t)fused_layout(d, nff).total; }

cudaError_t launch_fused(const FusedArgs &a, cudaStream_t s, int n_sms) {
    FusedParams p{};
    p.w_router = a.w_router; p.b_router = a.b_router; p.x = a.x;
    p.nrm = a.nrm; p.nsum = a.nsum;
    p.T = a.T; p.E = a.E; p.d = a.d; p.k = a.k; p.nff = a.nff;
    p.res = a.res;
    p.hot_gu = a.hot_gu; p.cold_gu = a.cold_gu; p.hot_dn = a.hot_dn; p.cold_dn = a.cold_dn;
    p.logits = a.logits; p.xq = a.xq; p.xq_stride = a.xq_stride;
    p.h = a.h; p.y = a.y; p.out = a.out;
    p.ids_out = a.ids_out; p.w_out = a.w_out; p.cnt_out = a.cnt_out; p.off_out = a.off_out; p.perm_out = a.perm_out;
    p.qa = a.qa;
    p.sync = a.sync;
    const size_t smem = fused_smem_bytes(a.d, a.nff);
    const void *fn = a.nrm.pre ? (const void *)fused_decode_kernel<true> : (const void *)fused_decode_kernel<false>;
    static unsigned optin[32];   // per device: the attribute belongs to each device's context
    const cudaError_t e = smem_optin(fn, 227 * 1024, optin, a.nrm.pre ? 1 : 0);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_sms);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // the grid barriers need every CTA resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&p};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Optional per-kernel CUDA events around the nine prefill launches (moeb_prefill_profile).
namespace {
struct PfProfile {
    cudaEvent_t ev[kPrefillKernels + 1] = {};
    bool recorded = false;
};
std::atomic<bool> g_pf_prof_on{false};
std::mutex g_pf_prof_mu;
PfProfile g_pf_prof[32];
}  // namespace

static cudaError_t prof_mark(cudaStream_t s, int i) {
    if (!g_pf_prof_on.load(std::memory_order_relaxed)) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 32) return e;
    std::lock_guard<std::mutex> lk(g_pf_prof_mu);
    PfProfile &pp = g_pf_prof[dev];
    if (!pp.ev[i]) {
        e = cudaEventCreate(&pp.ev[i]);
        if (e != cudaSuccess) return e;
    }
    if (i == kPrefillKernels) pp.recorded = true;
    return cudaEventRecord(pp.ev[i], s);
}

int prefill_profile_read(float *ms, int n) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 32) return -1;
    std::lock_guard<std::mutex> lk(g_pf_prof_mu);
    PfProfile &pp = g_pf_prof[dev];
    if (!pp.recorded) return -1;
    if (cudaEventSynchronize(pp.ev[kPrefillKernels]) != cudaSuccess) return -1;
    for (int i = 0; i < n && i < kPrefillKernels; ++i)
        if (cudaEventElapsedTime(&ms[i], pp.ev[i], pp.ev[i + 1]) != cudaSuccess) return -1;
    return 0;
}

void prefill_profile_enable(bool on) { g_pf_prof_on.store(on); }

// launch_ex that, on failure, records which kernel failed and its compiled resource needs
static cudaError_t pf_launch(const char *name, const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             bool pdl, void **args) {
    cudaError_t e = launch_ex(fn, grid, block, smem, s, pdl, args);
    if (e != cudaSuccess) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, fn);
        set_last_error(MOEB_ECUDA, "%s launch (grid %u, block %u, dynamic smem %zu): %s [regs %d, max threads %d, "
                                   "static smem %zu, max dynamic smem %d]",
                       name, grid.x * grid.y, block.x, smem, cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock,
                       fa.sharedSizeBytes, fa.maxDynamicSharedSizeBytes);
    }
    return e;
}

bool mid_shape_ok(int kind, int d, int nff, int P, int E) {
    const int tiles = prefill_max_tiles(P, E);
    // n_ff <= 1024: the widths the mid-size kernels are tested at (wider layers take the tcgen05 GEMMs)
    return d % QK_K == 0 && nff % QK32 == 0 && nff <= 1024 && tiles <= kMdMaxTiles &&
           P / (8 * md_chunk(kind)) + tiles <= kMdMaxUnits && md_layout(kind, d, nff).n_slots >= 2;
}

// 2D tensor map of a Q4_K gate_up pool (row bytes x rows, one super-block x 64 rows per box) for the
// lane-exact gate_up kernel's raw-row staging; other pool types leave the map zero (unused)
static cudaError_t lx_encode_map(CUtensorMap *map, const PoolView &pv, int d, int nff) {
    std::memset(map, 0, sizeof(*map));
    if (!pv.w || pv.type != T_Q4_K || pv.n <= 0) return cudaSuccess;
    using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static Encode encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorNotSupported;
        encode = reinterpret_cast<Encode>(fn);
    }
    const cuuint64_t rb = (cuuint64_t)row_bytes(T_Q4_K, d);
    const cuuint64_t dims[2] = {rb, (cuuint64_t)pv.n * 2 * nff};
    const cuuint64_t strides[1] = {rb};
    const cuuint32_t box[2] = {(cuuint32_t)B_Q4_K, 64u};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(pv.w), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_prefill(const PrefillArgs &a, cudaStream_t s, int n_sms) {
    static unsigned optin[32];
    cudaError_t e = smem_optin((const void *)pf_gate_up_lx_kernel, sizeof(LxSmem), optin, 0);
    if (e == cudaSuccess) e = smem_optin((const void *)pf_down_kernel, sizeof(DnSmem), optin, 1);
    if (e == cudaSuccess) e = smem_optin((const void *)pf_q4k_min_kernel, min_smem_bytes(kPrefillMaxSb), optin, 4);
    if (e != cudaSuccess) return e;
    const int T = a.T, E = a.E, d = a.d, k = a.k;
    int mark = 0;
    if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    const bool nrm = a.nrm.pre != nullptr;
    if (nrm) {
        // the Gemma-4 block norms: row scales and the expert input's Q8_K rows in one kernel ahead of
        // the router (its time lands in the router's profile slot; the actq slot reads zero)
        const float *x = a.x, *pre = a.nrm.pre;
        int8_t *q = a.xq8;
        float *xd = a.xd, *ns = a.nscale;
        int16_t *bs = a.xbs;
        int t = T, dd = d;
        float eps = a.nrm.eps;
        void *args[] = {&x, &q, &xd, &bs, &ns, &pre, &t, &dd, &eps};
        e = pf_launch("pf_actq_norm_kernel", (const void *)pf_actq_norm_kernel, dim3(T), dim3((d / QK_K) * 32), 0, s,
                      true, args);
        if (e != cudaSuccess) return e;
    }
    if (!a.routed) {
        {
            const float *W = a.w_router, *x = a.x;
            float *part = a.rpart;
            int t = T, ne = E, dd = d, ns = router_splits(T, E, d);
            const float *nsc = nrm ? a.nscale : nullptr, *rsc = a.nrm.router;
            void *args[] = {&W, &x, &part, &t, &ne, &dd, &ns, &nsc, &rsc};
            e = pf_launch("pf_router_kernel", (const void *)pf_router_kernel,
                          dim3((T + kRtTok - 1) / kRtTok, ns, (E + kRtExp - 1) / kRtExp), dim3(256), 0, s, true, args);
            if (e != cudaSuccess) return e;
            if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        }
        {
            const float *part = a.rpart, *b = a.b_router;
            float *lg = a.logits;
            int32_t *ids = a.ids;
            float *w = a.w;
            int t = T, ne = E, kk = k, ns = router_splits(T, E, d);
            void *args[] = {&part, &b, &lg, &ids, &w, &t, &ne, &kk, &ns};
            e = pf_launch("pf_topk_kernel", (const void *)pf_topk_kernel, dim3((T + 7) / 8), dim3(256), 0, s, true, args);
            if (e != cudaSuccess) return e;
            if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        }
    } else {   // routing given: the router and top-k slots of the profile read zero
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    }
    {
        PfDispatchParams dp{};
        dp.ids = a.ids; dp.T = T; dp.E = E; dp.k = k;
        dp.res = a.res;
        dp.hot_n = a.hot_gu.w ? a.hot_gu.n : 0;
        dp.cold_n = a.cold_gu.w ? a.cold_gu.n : 0;
        dp.cnt = a.cnt; dp.off = a.off; dp.perm = a.perm; dp.pos = a.pos;
        dp.tiles = a.tiles; dp.n_tiles = a.n_tiles;
        void *args[] = {&dp};
        e = pf_launch("pf_dispatch_kernel", (const void *)pf_dispatch_kernel, dim3(1), dim3(1024), 0, s, true, args);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    }
    if (!nrm && a.xq_rows) {
        const uint8_t *rows = a.xq_rows;
        int8_t *q = a.xq8;
        float *xd = a.xd;
        int16_t *bs = a.xbs;
        int t = T, dd = d;
        void *args[] = {&rows, &q, &xd, &bs, &t, &dd};
        e = pf_launch("pf_unpack_q8k_kernel", (const void *)pf_unpack_q8k_kernel, dim3((T * (d / QK_K) + 7) / 8), dim3(256),
                      0, s, true, args);
        if (e != cudaSuccess) return e;
    } else if (!nrm) {
        const float *x = a.x;
        int8_t *q = a.xq8;
        float *xd = a.xd;
        int16_t *bs = a.xbs;
        int t = T, dd = d;
        void *args[] = {&x, &q, &xd, &bs, &t, &dd};
        e = pf_launch("pf_actq_kernel", (const void *)pf_actq_kernel, dim3((T * (d / QK_K) + 7) / 8), dim3(256), 0, s, true, args);
        if (e != cudaSuccess) return e;
    }
    if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    // gate_up and down each run the mid-size kernels (mid.cuh) or the tcgen05 kernels; both write the
    // gate_up rows to hbuf in slot order, so the two choices are independent
    MdParams m{};
    m.T = T; m.E = E; m.d = d; m.k = k; m.nff = a.nff;
    m.tiles = a.tiles; m.n_tiles = a.n_tiles; m.perm = a.perm; m.img = a.bimg;
    if (a.mid_gu || a.mid_dn) {
        // opt in once at the largest size any layer shape may ask for
        e = smem_optin((const void *)md_kernel<0>, 227 * 1024, optin, 2);
        if (e == cudaSuccess) e = smem_optin((const void *)md_kernel<1>, 227 * 1024, optin, 3);
        if (e != cudaSuccess) return e;
    }
    PfParams p{};
    p.T = T; p.E = E; p.d = d; p.k = k; p.nff = a.nff;
    p.gu[0] = a.hot_gu; p.gu[1] = a.cold_gu; p.dn[0] = a.hot_dn; p.dn[1] = a.cold_dn;
    p.perm = a.perm; p.tiles = a.tiles; p.n_tiles = a.n_tiles;
    p.xq8 = a.xq8; p.xd = a.xd; p.xbs = a.xbs;
    p.bimg = a.bimg; p.dxt = a.dxt; p.bst = a.bst; p.hbuf = a.hbuf; p.dimg = a.dimg; p.h = a.h; p.y = a.y;
    void *pargs[] = {&p};
    if (a.mid_gu) {
        {
            const PfTile *tl = a.tiles;
            const int32_t *nt = a.n_tiles, *perm = a.perm;
            const int8_t *q = a.xq8;
            const float *xd = a.xd;
            const int16_t *bs = a.xbs;
            uint8_t *img = a.bimg;
            int kk = k, dd = d;
            void *args[] = {&tl, &nt, &perm, &q, &xd, &bs, &img, &kk, &dd};
            e = pf_launch("md_bimg_kernel", (const void *)md_bimg_kernel, dim3(a.md_max_cb, d / QK_K), dim3(256), 0, s,
                          true, args);
            if (e != cudaSuccess) return e;
            if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        }
        m.pv[0] = a.hot_gu; m.pv[1] = a.cold_gu; m.out = a.hbuf;
        void *args[] = {&m};
        e = pf_launch("md_kernel<0>", (const void *)md_kernel<0>, dim3(n_sms), dim3(kMdThreads),
                      (size_t)md_layout(0, d, a.nff).total, s, true, args);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    } else {
        e = pf_launch("pf_gather_lx_kernel", (const void *)pf_gather_lx_kernel, dim3(a.max_tiles, d / QK_K), dim3(256), 0,
                      s, true, pargs);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        // the Q4_K min term of every (row, pair) into hbuf, which the grouped GEMM's epilogue completes
        // (both run inside the gate_up profile slot)
        e = pf_launch("pf_q4k_min_kernel", (const void *)pf_q4k_min_kernel,
                      dim3(a.max_tiles, 2 * a.nff / kMinRows), dim3(kMinThreads), min_smem_bytes(d / QK_K), s, true,
                      pargs);
        if (e != cudaSuccess) return e;
        LxMaps maps;
        if ((e = lx_encode_map(&maps.gu[0], a.hot_gu, d, a.nff)) != cudaSuccess) return e;
        if ((e = lx_encode_map(&maps.gu[1], a.cold_gu, d, a.nff)) != cudaSuccess) return e;
        void *largs[] = {&p, &maps};
        e = pf_launch("pf_gate_up_lx_kernel", (const void *)pf_gate_up_lx_kernel, dim3(n_sms), dim3(kLxThreads),
                      sizeof(LxSmem), s, true, largs);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    }
    if (a.mid_dn) {
        {
            const PfTile *tl = a.tiles;
            const int32_t *nt = a.n_tiles, *perm = a.perm;
            const float *hb = a.hbuf;
            uint8_t *img = a.bimg;
            float *hp = a.h;
            int nf = a.nff;
            void *args[] = {&tl, &nt, &perm, &hb, &img, &hp, &nf};
            e = pf_launch("md_act_kernel", (const void *)md_act_kernel, dim3(a.md_max_cb, (a.nff / QK32 + 7) / 8), dim3(256),
                          0, s, true, args);
            if (e != cudaSuccess) return e;
            if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        }
        m.pv[0] = a.hot_dn; m.pv[1] = a.cold_dn; m.out = a.y;
        void *args[] = {&m};
        e = pf_launch("md_kernel<1>", (const void *)md_kernel<1>, dim3(n_sms), dim3(kMdThreads),
                      (size_t)md_layout(1, d, a.nff).total, s, true, args);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    } else {
        e = pf_launch("pf_geglu_kernel", (const void *)pf_geglu_kernel, dim3(a.max_tiles, a.nff / 32), dim3(256), 0, s,
                      true, pargs);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
        e = pf_launch("pf_down_kernel", (const void *)pf_down_kernel, dim3(n_sms), dim3(kDnThreads), sizeof(DnSmem), s, true,
                      pargs);
        if (e != cudaSuccess) return e;
        if ((e = prof_mark(s, mark++)) != cudaSuccess) return e;
    }
    {
        const float *y = a.y, *w = a.w;
        const int32_t *pos = a.pos;
        float *out = a.out, *yp = a.y_pairs;
        int t = T, kk = k, dd = d;
        const float *post = nrm ? a.nrm.post : nullptr;
        float eps = a.nrm.eps;
        void *args[] = {&y, &pos, &w, &out, &yp, &t, &kk, &dd, &post, &eps};
        e = pf_launch("pf_combine_kernel", (const void *)pf_combine_kernel, dim3(T), dim3(kCbThreads), 0, s, true, args);
        if (e != cudaSuccess) return e;
    }
    return prof_mark(s, mark++);
}

cudaError_t launch_route(const float *w_router, const float *b_router, const float *x, int T, int E, int d, int k,
                         float *part, float *logits, int32_t *ids, float *w, cudaStream_t s) {
    // with `part` the K split is four-way into it; without, one part straight into the logits
    // buffer, which the top-k kernel completes in place (bias)
    int t = T, ne = E, dd = d, kk = k, ns = part ? kRtSplit : 1;
    float *dst = part ? part : logits;
    const float *no_norm = nullptr;
    void *a1[] = {&w_router, &x, &dst, &t, &ne, &dd, &ns, &no_norm, &no_norm};
    cudaError_t e = pf_launch("pf_router_kernel", (const void *)pf_router_kernel,
                              dim3((T + kRtTok - 1) / kRtTok, ns, (E + kRtExp - 1) / kRtExp), dim3(256), 0, s, true, a1);
    if (e != cudaSuccess) return e;
    const float *pc = dst;
    void *a2[] = {&pc, &b_router, &logits, &ids, &w, &t, &ne, &kk, &ns};
    return pf_launch("pf_topk_kernel", (const void *)pf_topk_kernel, dim3((T + 7) / 8), dim3(256), 0, s, true, a2);
}

__global__ void sum4_kernel(const float *h, size_t stride, float *dst, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __fadd_rn(__fadd_rn(__fadd_rn(h[i], h[i + stride]), h[i + 2 * stride]), h[i + 3 * stride]);
}

cudaError_t launch_sum4(const float *h, size_t stride, float *dst, size_t n, cudaStream_t s) {
    sum4_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(h, stride, dst, n);
    return cudaGetLastError();
}

// Row-wise rms_norm with the reference nodes that follow it (gemma4.cpp:394-402, :423-425):
// out = ((x * s) * c) * w, s = 1 / sqrt(mean(x^2) + eps), each product rounded to f32 as the separate
// rms_norm, scale (when c != 1) and mul (when w is given) nodes round it. One CTA per row; the squares
// are rounded to f32 and summed in double, as in the layer kernels' fused norms.
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *x, const float *w, float c, float eps, float *out,
                                                       int d) {
    __shared__ double red[8];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, n4 = d / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)row * d);
    double q = 0.0;
    for (int i = tid; i < n4; i += 256) q += sq_sum4(__ldg(x4 + i));
    q = warp_sum_d(q);
    if (lane == 0) red[warp] = q;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < 8; ++i) tot += red[i];   // one fixed order, every thread the same scale
    const float sc = rms_row_scale(tot, d, eps);
    float4 *o4 = reinterpret_cast<float4 *>(out + (size_t)row * d);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    for (int i = tid; i < n4; i += 256) {
        const float4 v = __ldg(x4 + i);
        float4 r = make_float4(__fmul_rn(v.x, sc), __fmul_rn(v.y, sc), __fmul_rn(v.z, sc), __fmul_rn(v.w, sc));
        if (c != 1.f) r = make_float4(__fmul_rn(r.x, c), __fmul_rn(r.y, c), __fmul_rn(r.z, c), __fmul_rn(r.w, c));
        if (w) {
            const float4 g = __ldg(w4 + i);
            r = make_float4(__fmul_rn(r.x, g.x), __fmul_rn(r.y, g.y), __fmul_rn(r.z, g.z), __fmul_rn(r.w, g.w));
        }
        o4[i] = r;
    }
}

cudaError_t launch_rms_norm(const float *x, int rows, int d, const float *w, float c, float eps, float *out,
                            cudaStream_t s) {
    rms_norm_kernel<<<rows, 256, 0, s>>>(x, w, c, eps, out, d);
    return cudaGetLastError();
}

// out += a (f32, n a multiple of 4, 16-byte aligned): the Gemma-4 block's ggml_add of the MoE and
// dense-MLP branches (gemma4.cpp:429), one rounding per element like the reference's
__global__ void add_f32_kernel(float4 *out, const float4 *a, size_t n4) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 o = out[i];
        const float4 v = __ldg(a + i);
        o.x = __fadd_rn(o.x, v.x);
        o.y = __fadd_rn(o.y, v.y);
        o.z = __fadd_rn(o.z, v.z);
        o.w = __fadd_rn(o.w, v.w);
        out[i] = o;
    }
}

cudaError_t launch_add_f32(float *out, const float *a, size_t n, int n_sms, cudaStream_t s) {
    const size_t n4 = n / 4;
    const size_t want = (n4 + 255) / 256, cap = (size_t)(n_sms > 0 ? n_sms : 148) * 8;
    add_f32_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, s>>>(reinterpret_cast<float4 *>(out),
                                                                        reinterpret_cast<const float4 *>(a), n4);
    return cudaGetLastError();
}

cudaError_t launch_quant_q8k(const float *x, uint8_t *dst, int rows, int d, int stride, cudaStream_t s) {
    quant_q8k_kernel<<<rows, kThreads, 0, s>>>(x, dst, d, stride);
    return cudaGetLastError();
}

cudaError_t launch_route_only(const RouteSrc &r, int32_t *ids, float *w, int32_t *cnt, int32_t *off, int32_t *perm,
                              cudaStream_t s) {
    route_only_kernel<<<1, kThreads, 0, s>>>(r, ids, w, cnt, off, perm);
    return cudaGetLastError();
}

cudaError_t launch_dequant(int32_t type, const void *src, float *dst, int64_t rows, int64_t n, cudaStream_t s) {
    const int64_t items = rows * (n / 32);
    dequant_kernel<<<(unsigned)((items + 127) / 128), 128, 0, s>>>(type, (const uint8_t *)src, dst, rows, n);
    return cudaGetLastError();
}

cudaError_t launch_quant_act(int32_t vdt, const float *x, void *dst, int64_t rows, int64_t n, cudaStream_t s) {
    quant_act_kernel<<<(unsigned)rows, kThreads, 0, s>>>(vdt, x, (uint8_t *)dst, n);
    return cudaGetLastError();
}

cudaError_t upload_gelu_table(const uint16_t *host_table, cudaStream_t s) {
    return cudaMemcpyToSymbolAsync(g_gelu_f16, host_table, sizeof(uint16_t) << 16, 0, cudaMemcpyHostToDevice, s);
}

cudaError_t read_and_clear_error(int32_t *out, cudaStream_t s) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_error, sizeof(int32_t), 0, cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return e;
    const int32_t zero = 0;
    e = cudaMemcpyToSymbolAsync(g_error, &zero, sizeof(int32_t), 0, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return e;
    if (*out & ERR_GRID_TIMEOUT) {
        // a CTA gave up a grid barrier: the barrier word may hold a partial count; the launch has
        // ended (stream order), so start the next one from zero
        const unsigned zw = 0;
        e = cudaMemcpyToSymbolAsync(g_bar_word, &zw, sizeof(unsigned), 0, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
    }
    return cudaStreamSynchronize(s);
}


// ------------------------------------------------------------------ allocation-free layer entry
// moeb_layer_forward_static(): the whole-layer forward with its workspace in this module-scope
// array instead of caller memory, for hosts that cannot allocate device memory on the call path
// (see include/moeb200.h). Every device that loads the library holds this array until exit.
static __device__ __align__(256) uint8_t g_static_scratch[MOEB_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_mu;
void *g_static_addr[64];   // device address of g_static_scratch, per device, resolved once
}  // namespace

}  // namespace moeb

#ifdef MOEB_TRACE
extern "C" int moeb_trace_read(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, moeb::g_ftrace, bytes) == cudaSuccess ? 0 : -3;
}
extern "C" int moeb_strace_read(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, moeb::g_strace, bytes) == cudaSuccess ? 0 : -3;
}
extern "C" int moeb_ptrace_read(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, moeb::g_ptrace, bytes) == cudaSuccess ? 0 : -3;
}
extern "C" int moeb_mdtrace_read(void *host, size_t bytes, void *host_u, size_t bytes_u) {
    if (cudaMemcpyFromSymbol(host, moeb::g_mdtrace, bytes) != cudaSuccess) return -3;
    return cudaMemcpyFromSymbol(host_u, moeb::g_mdutrace, bytes_u) == cudaSuccess ? 0 : -3;
}
extern "C" int moeb_xtrace_read(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, moeb::g_xtrace, bytes) == cudaSuccess ? 0 : -3;
}
extern "C" int moeb_utrace_read(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, moeb::g_utrace, bytes) == cudaSuccess ? 0 : -3;
}
#endif

extern "C" int moeb_layer_forward_static(const moeb_layer *L, const float *x, int32_t n_tokens, float *out,
                                         void *stream) {
    using namespace moeb;
    const size_t need = chunk_workspace_size(L, n_tokens);
    if (n_tokens > 0 && need > MOEB_STATIC_SCRATCH_BYTES)
        return set_last_error(MOEB_ESPACE, "moeb_layer_forward_static: this layer needs a %zu-byte workspace; the "
                                           "static scratch holds %u bytes (use moeb_layer_forward)",
                              need, (unsigned)MOEB_STATIC_SCRATCH_BYTES);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64)
        return set_last_error(MOEB_ENODEV, "moeb_layer_forward_static: no usable CUDA device");
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_static_mu);
        if (!g_static_addr[dev]) {
            // In host code g_static_scratch names a host-side shadow, not device memory: the kernels
            // need the device address, looked up once per device with that device current.
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess || !p)
                return set_last_error(MOEB_ECUDA, "moeb_layer_forward_static: cudaGetSymbolAddress failed: %s",
                                      cudaGetErrorString(e));
            g_static_addr[dev] = p;
        }
        scratch = g_static_addr[dev];
    }
    // Every byte of the workspace the forward reads is written earlier in the same forward, so the
    // previous call's contents need no clearing.
    return layer_forward_chunked(L, x, n_tokens, out, scratch, MOEB_STATIC_SCRATCH_BYTES, stream);
}
