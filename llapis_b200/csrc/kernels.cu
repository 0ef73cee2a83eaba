// Decode-size MoE layer kernels for sm_100a.
//
//   router_kernel   : router logits (f32 GEMV, one CTA per expert, fixed reduction order) + bias,
//                     and the Q8_K quantisation of every token (extra CTAs).
//   gemv_kernel     : grouped GEMV over the routed experts for one projection. Every CTA redoes
//                     the routing (softmax / top-k / weights) and the dispatch (histogram, exclusive
//                     scan, stable permutation) in shared memory from the logits, splits the routed
//                     experts' weight bytes evenly over the grid, streams its share HBM -> shared
//                     memory with bulk async copies (multi-stage mbarrier ring), and decodes the
//                     quantised blocks in registers into integer dp4a dot products with per-block
//                     float scaling — the same integer work as ggml-cpu's vec_dot kernels.
//                     kind 0: gate_up (Q4_K / IQ2_S weights, Q8_K activations).
//                     kind 1: down, activations = GeGLU(gate_up) quantised to Q8_0 in the prologue.
//                     kind 2: down, activations given (the moert per-kind ABI).
//   combine_kernel  : routing-weighted sum over the top-k slots in slot order.
// Kernels are chained with programmatic dependent launch: the down GEMV starts streaming its
// weights while the gate_up GEMV is still running, and only then waits for the gate_up outputs.
#include "common.cuh"

#include <algorithm>
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
__device__ void q8k_superblock_warp(const float *x, int8_t *qs, float *d_out, int16_t *bs, int lane) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[lane * 8 + i];
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

// ------------------------------------------------------------------ router
__global__ void __launch_bounds__(kThreads) router_kernel(RouterParams p) {
    // let the dependent GEMV grid start its table prologue while the router runs
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.x;
    if (b < p.E) {
        __shared__ float red[kMaxDecodeT][kWarps];
        const int n4 = p.d / 4;
        const float4 *w4 = reinterpret_cast<const float4 *>(p.w_router + (size_t)b * p.d);
        float part[kMaxDecodeT];
#pragma unroll
        for (int t = 0; t < kMaxDecodeT; ++t) part[t] = 0.f;
        for (int i = tid; i < n4; i += kThreads) {
            const float4 w = __ldg(w4 + i);
#pragma unroll
            for (int t = 0; t < kMaxDecodeT; ++t) {
                if (t < p.T) {
                    const float4 xv = reinterpret_cast<const float4 *>(p.x + (size_t)t * p.d)[i];
                    part[t] = fmaf(w.x, xv.x, part[t]);
                    part[t] = fmaf(w.y, xv.y, part[t]);
                    part[t] = fmaf(w.z, xv.z, part[t]);
                    part[t] = fmaf(w.w, xv.w, part[t]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kMaxDecodeT; ++t) {
            if (t < p.T) {
                const float s = warp_sum(part[t]);
                if (lane == 0) red[t][warp] = s;
            }
        }
        __syncthreads();
        if (tid < p.T) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s += red[tid][w];
            if (p.b_router) s = __fadd_rn(s, p.b_router[b]);
            p.logits[(size_t)tid * p.E + b] = s;
        }
    } else if (p.xq) {
        const int t = b - p.E;
        const int nsb = p.d / QK_K;
        uint8_t *row = p.xq + (size_t)t * p.xq_stride;
        int8_t *qs = reinterpret_cast<int8_t *>(row);
        float *dd = reinterpret_cast<float *>(row + nsb * 256);
        int16_t *bs = reinterpret_cast<int16_t *>(row + nsb * 256 + nsb * 4);
        for (int sb = warp; sb < nsb; sb += kWarps)
            q8k_superblock_warp(p.x + (size_t)t * p.d + sb * 256, qs + sb * 256, dd + sb, bs + sb * 16, lane);
    }
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
__device__ void route_tokens(const RouteSrc &r, RouteSmem &rs, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    const int per = r.E / 32;
    for (int t = warp; t < r.T; t += kWarps) {
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
                               int d_in, int d_out, RouteSmem &rs, int tid, bool check_pools) {
    const int P = r.T * r.k;
    for (int e = tid; e < r.E; e += kThreads) rs.cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += kThreads) {
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
    for (int p = tid; p < P; p += kThreads) {
        const int e = rs.ids[p];
        int rank = 0;
        for (int q = 0; q < p; ++q) rank += rs.ids[q] == e;
        rs.perm[rs.off[e] + rank] = p;
    }
    __syncthreads();
}

// ------------------------------------------------------------------ per-format row dot products
// Each returns, for one lane, its partial contribution to rows' dot products with up to
// kTokChunk activation columns; the caller sums the lanes that share a row.

// IQ2_S x Q8_K: lane owns 32-value sub-block j of every super-block (8 lanes per row).
// Integer part per sub-block: ls0*sum(l=0,1) + ls1*sum(l=2,3) with ls = 1 + 2*nibble; float:
// (d_w * d_x) per super-block; the caller scales the total by 0.125 (ggml-cpu/quants.c:947-990).
__device__ __forceinline__ void dot_iq2s_lane(const uint8_t *row, int nsb, int j, const uint64_t *grid,
                                              const uint8_t *act, int act_stride, const int *tok, int ntok,
                                              float *acc) {
    for (int sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + sb * B_IQ2_S;
        const float dw = h2f(ld_u16(blk));
        const uint32_t qs4 = ld_u32_a2(blk + 2 + 4 * j);
        const uint32_t sg4 = ld_u32_a2(blk + 34 + 4 * j);
        const uint32_t qh = blk[66 + j];
        const uint32_t sc = blk[74 + j];
        int wv[8];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t gi = ((qs4 >> (8 * l)) & 0xffu) | (((qh >> (2 * l)) & 3u) << 8);
            const uint64_t g = grid[gi];
            const uint32_t s = (sg4 >> (8 * l)) & 0xffu;
            const uint32_t c0 = ((s & 15u) * 0x00204081u) & 0x01010101u;
            const uint32_t c1 = ((s >> 4) * 0x00204081u) & 0x01010101u;
            // negate the flagged bytes: (w ^ 0xff) + 1 == -w, and magnitudes >= 8 never carry
            wv[2 * l] = (int)(((uint32_t)g ^ (c0 * 0xffu)) + c0);
            wv[2 * l + 1] = (int)(((uint32_t)(g >> 32) ^ (c1 * 0xffu)) + c1);
        }
        const int ls0 = 1 + 2 * (int)(sc & 15u), ls1 = 1 + 2 * (int)(sc >> 4);
#pragma unroll
        for (int c = 0; c < kTokChunk; ++c) {
            if (c < ntok) {
                const Q8KView xv = q8k_view(act + (size_t)tok[c] * act_stride, nsb);
                const int4 *q = reinterpret_cast<const int4 *>(xv.qs + sb * 256 + 32 * j);
                const int4 qa = q[0], qb = q[1];
                int s0 = dp4a(wv[0], qa.x, 0);
                s0 = dp4a(wv[1], qa.y, s0);
                s0 = dp4a(wv[2], qa.z, s0);
                s0 = dp4a(wv[3], qa.w, s0);
                int s1 = dp4a(wv[4], qb.x, 0);
                s1 = dp4a(wv[5], qb.y, s1);
                s1 = dp4a(wv[6], qb.z, s1);
                s1 = dp4a(wv[7], qb.w, s1);
                acc[c] += (dw * xv.d[sb]) * (float)(ls0 * s0 + ls1 * s1);
            }
        }
    }
}

// Q4_K x Q8_K: lane owns sub-block j (32 values) of every super-block (8 lanes per row).
// main = s_j * sum(q4 * q8), min = m_j * (bsum[2j] + bsum[2j+1]);
// float (d_w d_x) main - (dmin_w d_x) min (ggml-cpu/quants.c:645-715).
__device__ __forceinline__ void dot_q4k_lane(const uint8_t *row, int nsb, int j, const uint8_t *act, int act_stride,
                                             const int *tok, int ntok, float *acc) {
    for (int sb = 0; sb < nsb; ++sb) {
        const uint8_t *blk = row + sb * B_Q4_K;
        const uint32_t dm = *reinterpret_cast<const uint32_t *>(blk);
        const float dw = h2f((uint16_t)(dm & 0xffffu)), dmin = h2f((uint16_t)(dm >> 16));
        const uint8_t *sc = blk + 4;
        int s, m;
        if (j < 4) {
            s = sc[j] & 63;
            m = sc[j + 4] & 63;
        } else {
            s = (sc[j + 4] & 0x0f) | ((sc[j - 4] >> 6) << 4);
            m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
        const int4 *qp = reinterpret_cast<const int4 *>(blk + 16 + 32 * (j >> 1));
        const int4 qa = qp[0], qb = qp[1];
        const int sh = 4 * (j & 1);
        int wv[8];
        wv[0] = (qa.x >> sh) & 0x0f0f0f0f; wv[1] = (qa.y >> sh) & 0x0f0f0f0f;
        wv[2] = (qa.z >> sh) & 0x0f0f0f0f; wv[3] = (qa.w >> sh) & 0x0f0f0f0f;
        wv[4] = (qb.x >> sh) & 0x0f0f0f0f; wv[5] = (qb.y >> sh) & 0x0f0f0f0f;
        wv[6] = (qb.z >> sh) & 0x0f0f0f0f; wv[7] = (qb.w >> sh) & 0x0f0f0f0f;
#pragma unroll
        for (int c = 0; c < kTokChunk; ++c) {
            if (c < ntok) {
                const Q8KView xv = q8k_view(act + (size_t)tok[c] * act_stride, nsb);
                const int4 *q = reinterpret_cast<const int4 *>(xv.qs + sb * 256 + 32 * j);
                const int4 xa = q[0], xb = q[1];
                int d = dp4a(wv[0], xa.x, 0);
                d = dp4a(wv[1], xa.y, d);
                d = dp4a(wv[2], xa.z, d);
                d = dp4a(wv[3], xa.w, d);
                d = dp4a(wv[4], xb.x, d);
                d = dp4a(wv[5], xb.y, d);
                d = dp4a(wv[6], xb.z, d);
                d = dp4a(wv[7], xb.w, d);
                const int bsum = xv.bs[sb * 16 + 2 * j] + xv.bs[sb * 16 + 2 * j + 1];
                const float dx = xv.d[sb];
                acc[c] += (dw * dx) * (float)(s * d);
                acc[c] -= (dmin * dx) * (float)(m * bsum);
            }
        }
    }
}

// Q8_0 activations in shared memory: qs[nb][32] int8 | d[nb] f32 (f16 value widened) | qsum[nb] i32
struct Q80View {
    const int8_t *qs;
    const float *d;
    const int *qsum;
};
__device__ __forceinline__ Q80View q80_view(const uint8_t *row, int nb) {
    Q80View v;
    v.qs = reinterpret_cast<const int8_t *>(row);
    v.d = reinterpret_cast<const float *>(row + nb * 32);
    v.qsum = reinterpret_cast<const int *>(row + nb * 36);
    return v;
}

// Q5_0 x Q8_0: lane owns half of a row's 32-blocks. value = (nibble | hbit << 4) - 16, so
// dot = sum(u * q) - 16 * sum(q); float d_w * d_x per block (ggml-cpu/quants.c:314-352).
__device__ __forceinline__ void dot_q5_0_lane(const uint8_t *row, int b0, int b1, const uint8_t *act, int act_stride,
                                              int nb, const int *col, int ntok, float *acc) {
    for (int b = b0; b < b1; ++b) {
        const uint8_t *blk = row + b * B_Q5_0;
        const float dw = h2f(ld_u16(blk));
        const uint32_t qh = ld_u32_a2(blk + 2);
        int wlo[4], whi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t q = ld_u32_a2(blk + 6 + 4 * i);
            const uint32_t hl = (((qh >> (4 * i)) & 15u) * 0x00204081u) & 0x01010101u;
            const uint32_t hh = (((qh >> (16 + 4 * i)) & 15u) * 0x00204081u) & 0x01010101u;
            wlo[i] = (int)((q & 0x0f0f0f0fu) | (hl << 4));
            whi[i] = (int)(((q >> 4) & 0x0f0f0f0fu) | (hh << 4));
        }
#pragma unroll
        for (int c = 0; c < kTokChunk; ++c) {
            if (c < ntok) {
                const Q80View xv = q80_view(act + (size_t)col[c] * act_stride, nb);
                const int4 *q = reinterpret_cast<const int4 *>(xv.qs + 32 * b);
                const int4 xa = q[0], xb = q[1];
                int s = dp4a(wlo[0], xa.x, 0);
                s = dp4a(wlo[1], xa.y, s);
                s = dp4a(wlo[2], xa.z, s);
                s = dp4a(wlo[3], xa.w, s);
                s = dp4a(whi[0], xb.x, s);
                s = dp4a(whi[1], xb.y, s);
                s = dp4a(whi[2], xb.z, s);
                s = dp4a(whi[3], xb.w, s);
                s -= 16 * xv.qsum[b];
                acc[c] += (dw * xv.d[b]) * (float)s;
            }
        }
    }
}

// 4 table lookups (IQ4_NL levels) for the 4 low nibbles of the bytes of `w`
__device__ __forceinline__ int iq4nl_lookup4(uint32_t w, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3) {
    const uint32_t x = w & 0x0f0f0f0fu;
    const uint32_t y = x | (x >> 4);
    const uint32_t sel = (y & 0xffu) | ((y >> 8) & 0xff00u);
    const uint32_t lo = __byte_perm(t0, t1, sel & 0x7777u);
    const uint32_t hi = __byte_perm(t2, t3, sel & 0x7777u);
    const uint32_t m = ((x >> 3) & 0x01010101u) * 0xffu;
    return (int)((lo & ~m) | (hi & m));
}

// IQ4_NL x Q8_0 (ggml-cpu/quants.c:1203-1227)
__device__ __forceinline__ void dot_iq4nl_lane(const uint8_t *row, int b0, int b1, const uint8_t *act, int act_stride,
                                               int nb, const int *col, int ntok, const uint32_t *kv, float *acc) {
    for (int b = b0; b < b1; ++b) {
        const uint8_t *blk = row + b * B_IQ4_NL;
        const float dw = h2f(ld_u16(blk));
        int wlo[4], whi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t q = ld_u32_a2(blk + 2 + 4 * i);
            wlo[i] = iq4nl_lookup4(q, kv[0], kv[1], kv[2], kv[3]);
            whi[i] = iq4nl_lookup4(q >> 4, kv[0], kv[1], kv[2], kv[3]);
        }
#pragma unroll
        for (int c = 0; c < kTokChunk; ++c) {
            if (c < ntok) {
                const Q80View xv = q80_view(act + (size_t)col[c] * act_stride, nb);
                const int4 *q = reinterpret_cast<const int4 *>(xv.qs + 32 * b);
                const int4 xa = q[0], xb = q[1];
                int s = dp4a(wlo[0], xa.x, 0);
                s = dp4a(wlo[1], xa.y, s);
                s = dp4a(wlo[2], xa.z, s);
                s = dp4a(wlo[3], xa.w, s);
                s = dp4a(whi[0], xb.x, s);
                s = dp4a(whi[1], xb.y, s);
                s = dp4a(whi[2], xb.z, s);
                s = dp4a(whi[3], xb.w, s);
                acc[c] += (xv.d[b] * dw) * (float)s;
            }
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
constexpr int kStages = 3;
constexpr int kGuStageRows = 32;     // 8 lanes per row, 4 rows per warp, 8 warps
constexpr int kDnStageRows = 128;    // 2 lanes per row, 16 rows per warp, 8 warps

struct StagePlan {
    int u, row0, nrows;
};

// the next stage from flat group f (8-row groups; every unique expert has gpe groups)
__device__ __forceinline__ StagePlan next_stage(int f, int g1, int gpe, int stage_groups) {
    StagePlan s;
    s.u = f / gpe;
    const int lg = f - s.u * gpe;
    int n = min(stage_groups, min(g1 - f, gpe - lg));
    s.row0 = lg * kGroupRows;
    s.nrows = n * kGroupRows;
    return s;
}

// flat group index of byte position `pos` in the unique-expert cost prefix
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


// Shared-memory layout of gemv_kernel (identical on host and device).
struct GemvSmem {
    int route, bars, grid, act, stage, stage_cap, total;
};
__host__ __device__ inline GemvSmem gemv_layout(int kind, int d_in, int T) {
    GemvSmem L;
    int o = 0;
    L.route = o; o += (int)((sizeof(RouteSmem) + 127) / 128 * 128);
    L.bars = o;  o += 128;
    L.grid = o;  o += kind == 0 ? MOE_IQ2S_GRID_ROWS * 8 : 0;
    L.act = o;   o += (kind == 0 ? T * xq_stride_bytes(d_in) : T * q80_stride(d_in) + 16);
    o = (o + 127) / 128 * 128;
    L.stage = o;
    L.stage_cap = kind == 0 ? kGuStageRows * (int)row_bytes(T_Q4_K, d_in) : kDnStageRows * (int)row_bytes(T_Q5_0, d_in);
    L.stage_cap = (L.stage_cap + 127) / 128 * 128;
    o += kStages * L.stage_cap;
    L.total = o;
    return L;
}

__device__ __forceinline__ const uint8_t *pool_entry(const PoolView &pv, int widx, int d_out, int d_in) {
    if (pv.ptrs) return reinterpret_cast<const uint8_t *>(pv.ptrs[widx]);
    return pv.w + (size_t)widx * d_out * row_bytes(pv.type, d_in);
}

__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const GemvSmem L = gemv_layout(p.kind == 0 ? 0 : 1, p.d_in, p.route.T);
    RouteSmem &rs = *reinterpret_cast<RouteSmem *>(smem + L.route);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint64_t *grid = reinterpret_cast<uint64_t *>(smem + L.grid);
    uint8_t *act = smem + L.act;
    uint8_t *stage = smem + L.stage;

    // ---- prologue independent of upstream results
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    if (p.kind == 0)
        for (int i = tid; i < MOE_IQ2S_GRID_ROWS; i += kThreads) grid[i] = g_iq2s_grid[i];
    uint32_t kv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        kv[i] = (uint32_t)(uint8_t)g_iq4nl[4 * i] | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 1] << 8) |
                ((uint32_t)(uint8_t)g_iq4nl[4 * i + 2] << 16) | ((uint32_t)(uint8_t)g_iq4nl[4 * i + 3] << 24);

    // gate_up reads the router's logits and Q8_K activations: wait for the router grid. The down
    // projection's routing inputs were complete before the gate_up grid got past its own wait, so it
    // routes and starts streaming weights first and waits for the gate_up outputs later.
    if (p.kind == 0) pdl_wait();
    __syncthreads();

    // ---- routing and dispatch (every CTA, identical results)
    route_tokens(p.route, rs, tid);
    __syncthreads();
    dispatch_pairs(p.route, p.res, p.hot, p.cold, p.d_in, p.d_out, rs, tid, true);
    const int T = p.route.T, k = p.route.k, P = T * k;
    if (blockIdx.x == 0) {
        for (int i = tid; i < P; i += kThreads) {
            if (p.ids_out) p.ids_out[i] = rs.ids[i];
            if (p.w_out) p.w_out[i] = rs.w[i];
            if (p.perm_out) p.perm_out[i] = rs.perm[i];
        }
        for (int e = tid; e <= p.route.E; e += kThreads) {
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

    // ---- this CTA's share of the routed experts' weight bytes, in 8-row groups
    const int gpe = p.d_out / kGroupRows;
    const long long total = rs.upre[rs.n_unique];
    const long long s0 = total * blockIdx.x / gridDim.x, s1 = total * (blockIdx.x + 1) / gridDim.x;
    const int g0 = group_at(rs, s0, gpe), g1 = group_at(rs, s1, gpe);
    const int stage_groups = (p.kind == 0 ? kGuStageRows : kDnStageRows) / kGroupRows;

    auto stage_src = [&](const StagePlan &st, int &bytes) -> const uint8_t * {
        const int cls = rs.ucls[st.u];
        const PoolView &pv = cls == 0 ? p.hot : p.cold;
        const int rb = (int)row_bytes(pv.type, p.d_in);
        bytes = st.nrows * rb;
        return pool_entry(pv, rs.uwidx[st.u], p.d_out, p.d_in) + (size_t)st.row0 * rb;
    };

    int f_issue = g0, issued = 0;
    if (tid == 0) {
        for (int s = 0; s < kStages && f_issue < g1; ++s) {
            const StagePlan st = next_stage(f_issue, g1, gpe, stage_groups);
            int bytes;
            const uint8_t *src = stage_src(st, bytes);
            mbar_expect_tx(&bars[s], (uint32_t)bytes);
            bulk_g2s(stage + s * L.stage_cap, src, (uint32_t)bytes, &bars[s]);
            f_issue += st.nrows / kGroupRows;
            ++issued;
        }
    }

    // ---- activations
    if (p.kind == 0) {
        const int n16 = T * p.xq_stride / 16;
        const int4 *src = reinterpret_cast<const int4 *>(p.xq);
        int4 *dst = reinterpret_cast<int4 *>(act);
        for (int i = tid; i < n16; i += kThreads) dst[i] = src[i];
    } else if (p.kind == 1) {
        pdl_wait();   // gate_up outputs
    }
    __syncthreads();

    const int nsb = p.d_in / QK_K, nb = p.d_in / QK32;
    const int a_stride = p.kind == 0 ? p.xq_stride : q80_stride(p.d_in);
    int cur_u = -1, it = 0;
    bool ok = true;
    for (int f = g0; f < g1;) {
        const StagePlan st = next_stage(f, g1, gpe, stage_groups);
        const int e = rs.uexp[st.u], cls = rs.ucls[st.u], widx = rs.uwidx[st.u];
        const int po = rs.off[e];
        int n = rs.cnt[e];
        if (p.kind != 0 && n > T) {
            // the down activation buffer holds one pair per token of an expert; an expert repeated
            // within a token's routes is reported and its extra pairs are not computed
            if (tid == 0) atomicOr(&g_error, ERR_CAPACITY);
            n = T;
        }
        if (p.kind != 0 && st.u != cur_u) {
            // Q8_0 activations of this expert's routed pairs: slot i <- pair perm[po + i]
            for (int item = warp; item < n * nb; item += kWarps) {
                const int i = item / nb, b = item - i * nb;
                const int pair = rs.perm[po + i];
                float v;
                if (p.kind == 1) {
                    const float *hp = p.h + (size_t)pair * 2 * p.d_in;
                    v = geglu1(hp[32 * b + lane], hp[p.d_in + 32 * b + lane]);
                } else {
                    v = p.a[(size_t)(p.a_per_pair ? pair : pair / k) * p.d_in + 32 * b + lane];
                }
                uint8_t *row = act + (size_t)i * a_stride;
                q80_block_warp(v, reinterpret_cast<int8_t *>(row) + 32 * b, reinterpret_cast<float *>(row + nb * 32) + b,
                               reinterpret_cast<int *>(row + nb * 36) + b, lane);
            }
            cur_u = st.u;
            __syncthreads();
        }
        const int buf = it % kStages;
        const uint32_t parity = (uint32_t)((it / kStages) & 1);
        if (!mbar_wait(&bars[buf], parity)) { ok = false; break; }
        const uint8_t *sb = stage + buf * L.stage_cap;
        const PoolView &pv = cls == 0 ? p.hot : p.cold;
        const int rb = (int)row_bytes(pv.type, p.d_in);
        if (p.kind == 0) {
            const int j = lane & 7, rsub = lane >> 3;
            for (int r0 = warp * 4; r0 < st.nrows; r0 += kWarps * 4) {
                const int r = r0 + rsub;
                const uint8_t *row = sb + (size_t)r * rb;
                for (int c0 = 0; c0 < n; c0 += kTokChunk) {
                    const int ntok = min(kTokChunk, n - c0);
                    int tok[kTokChunk], pair[kTokChunk];
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        pair[c] = c < ntok ? rs.perm[po + c0 + c] : 0;
                        tok[c] = pair[c] / k;
                    }
                    float acc[kTokChunk] = {0.f, 0.f, 0.f, 0.f};
                    if (pv.type == T_IQ2_S) dot_iq2s_lane(row, nsb, j, grid, act, a_stride, tok, ntok, acc);
                    else dot_q4k_lane(row, nsb, j, act, a_stride, tok, ntok, acc);
                    const float post = pv.type == T_IQ2_S ? 0.125f : 1.0f;
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        float v = acc[c];
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        v += __shfl_xor_sync(0xffffffffu, v, 2);
                        v += __shfl_xor_sync(0xffffffffu, v, 4);
                        if (j == 0 && c < ntok) p.y[(size_t)pair[c] * p.d_out + st.row0 + r] = v * post;
                    }
                }
            }
        } else {
            const int half = lane & 1, rsub = lane >> 1;
            const int bmid = (nb + 1) / 2;
            const int b0 = half ? bmid : 0, b1 = half ? nb : bmid;
            const float *scale = pv.scale;
            for (int r0 = warp * 16; r0 < st.nrows; r0 += kWarps * 16) {
                const int r = r0 + rsub;
                const bool valid = r < st.nrows;
                const uint8_t *row = sb + (size_t)(valid ? r : 0) * rb;
                for (int c0 = 0; c0 < n; c0 += kTokChunk) {
                    const int ntok = valid ? min(kTokChunk, n - c0) : 0;
                    int col[kTokChunk];
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) col[c] = c0 + c;
                    float acc[kTokChunk] = {0.f, 0.f, 0.f, 0.f};
                    if (pv.type == T_Q5_0) dot_q5_0_lane(row, b0, b1, act, a_stride, nb, col, ntok, acc);
                    else dot_iq4nl_lane(row, b0, b1, act, a_stride, nb, col, ntok, kv, acc);
#pragma unroll
                    for (int c = 0; c < kTokChunk; ++c) {
                        float v = acc[c];
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        if (half == 0 && c < ntok) {
                            const int pair = rs.perm[po + c0 + c];
                            if (p.apply_scale && scale) v = __fmul_rn(v, scale[widx]);
                            p.y[(size_t)pair * p.d_out + st.row0 + r] = v;
                        }
                    }
                }
            }
        }
        __syncthreads();   // every warp is done with this stage buffer
        if (tid == 0 && f_issue < g1) {
            const StagePlan nx = next_stage(f_issue, g1, gpe, stage_groups);
            int bytes;
            const uint8_t *src = stage_src(nx, bytes);
            mbar_expect_tx(&bars[buf], (uint32_t)bytes);
            bulk_g2s(stage + buf * L.stage_cap, src, (uint32_t)bytes, &bars[buf]);
            f_issue += nx.nrows / kGroupRows;
            ++issued;
        }
        f += st.nrows / kGroupRows;
        ++it;
    }
    if (!ok && tid == 0) {
        // a wait gave up: drain this CTA's copies still in flight (bounded) before leaving
        for (int i = it; i < issued; ++i) mbar_wait(&bars[i % kStages], (uint32_t)((i / kStages) & 1));
    }
}

// ------------------------------------------------------------------ combine
// out[t] = w[t][0]*y[t*k] + w[t][1]*y[t*k+1] + ...: products rounded, then added in slot order
// (ggml_mul then the view-add chain, llama-graph.cpp:1814-1848).
__global__ void __launch_bounds__(kThreads) combine_kernel(CombineParams p) {
    pdl_wait();
    const int t = blockIdx.y;
    const int i4 = blockIdx.x * kThreads + threadIdx.x;
    if (i4 * 4 >= p.d) return;
    float wj[kMaxTopK];
    for (int j = 0; j < p.k; ++j) wj[j] = p.w[t * p.k + j];
    const float4 *y4 = reinterpret_cast<const float4 *>(p.y);
    const int d4 = p.d / 4;
    float4 acc = y4[(size_t)(t * p.k) * d4 + i4];
    acc.x = __fmul_rn(acc.x, wj[0]); acc.y = __fmul_rn(acc.y, wj[0]);
    acc.z = __fmul_rn(acc.z, wj[0]); acc.w = __fmul_rn(acc.w, wj[0]);
    for (int j = 1; j < p.k; ++j) {
        const float4 v = y4[(size_t)(t * p.k + j) * d4 + i4];
        acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, wj[j]));
        acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, wj[j]));
        acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, wj[j]));
        acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, wj[j]));
    }
    reinterpret_cast<float4 *>(p.out)[(size_t)t * d4 + i4] = acc;
}

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
    route_tokens(r, rs, tid);
    __syncthreads();
    const Residency none = {0, nullptr, nullptr, nullptr};
    const PoolView pv = {nullptr, T_Q4_K, 0, nullptr};
    dispatch_pairs(r, none, pv, pv, QK_K, kGroupRows, rs, tid, false);
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
// them (ggml-quants.c:442,1471,2471,2653): no fused multiply-add.
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

cudaError_t launch_router(const RouterParams &p, cudaStream_t s, bool pdl) {
    RouterParams q = p;
    void *args[] = {&q};
    return launch_ex((const void *)router_kernel, dim3(p.E + (p.xq ? p.T : 0)), dim3(kThreads), 0, s, pdl, args);
}

size_t gemv_smem_bytes(int kind, int d_in, int T) { return (size_t)gemv_layout(kind == 0 ? 0 : 1, d_in, T).total; }

cudaError_t launch_gemv(const GemvParams &p, cudaStream_t s, bool pdl, int n_sms) {
    const size_t smem = gemv_smem_bytes(p.kind, p.d_in, p.route.T);
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute((const void *)gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    GemvParams q = p;
    void *args[] = {&q};
    return launch_ex((const void *)gemv_kernel, dim3(n_sms), dim3(kThreads), smem, s, pdl, args);
}

cudaError_t launch_combine(const CombineParams &p, cudaStream_t s, bool pdl) {
    CombineParams q = p;
    void *args[] = {&q};
    const int d4 = p.d / 4;
    return launch_ex((const void *)combine_kernel, dim3((d4 + kThreads - 1) / kThreads, p.T), dim3(kThreads), 0, s,
                     pdl, args);
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

extern "C" int moeb_layer_forward_static(const moeb_layer *L, const float *x, int32_t n_tokens, float *out,
                                         void *stream) {
    using namespace moeb;
    const size_t need = moeb_layer_workspace_size(L, n_tokens);
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
    return moeb_layer_forward(L, x, n_tokens, out, nullptr, scratch, MOEB_STATIC_SCRATCH_BYTES, stream);
}
