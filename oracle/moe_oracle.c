/*
 * TEST INFRASTRUCTURE — not product code.
 *
 * Plain-C restatement of the reference's CPU path for the Gemma-4 MoE FFN layer, written from the
 * reference's documented algorithm. It is the checker for the CUDA path; it is pinned against the
 * reference itself (oracle/_ref, built from the reference sources) and against the committed
 * golden fixtures in tests/golden/. Single-threaded, no SIMD. The quantised dot products restate the
 * float order of the reference's x86 kernels (8 lanes, fused multiply-add per block, the fixed
 * horizontal sum), so they are bit-equal to the reference's; every integer step (quantised
 * activations, routing indices) matches bit for bit. The f32 router logits are summed in double
 * here (the reference's f32 dot differs in the last bits; routing is compared off near ties).
 *
 * Each function cites the reference function it restates (paths relative to third_party/llama/ggml
 * unless stated).
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "ggml_tables.inc"

static const uint64_t k_iq2s_grid[MOE_IQ2S_GRID_ROWS] = MOE_IQ2S_GRID_INIT;
static const int8_t   k_iq4nl[16] = MOE_IQ4NL_VALUES_INIT;
static const uint64_t k_iq2xxs_grid[256] = MOE_IQ2XXS_GRID_INIT;
static const uint8_t  k_iq2xxs_signs[128] = MOE_IQ2XXS_SIGNS_INIT;

const uint64_t *oracle_iq2s_grid(void) { return k_iq2s_grid; }
const int8_t   *oracle_iq4nl_values(void) { return k_iq4nl; }

/* ------------------------------------------------------------------ half precision */

static float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> binary32, exact (what F16C's vcvtph2ps computes; src/ggml-impl.h:384). */
static float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ffu;
    if (e == 0x1f) return bits_f32(sign | 0x7f800000u | (m << 13));
    if (e == 0) {
        /* zero or subnormal: m * 2^-24 is exact in binary32 */
        const float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* binary32 -> binary16 with round-to-nearest-even (F16C vcvtps2ph imm 0). */
static uint16_t f2h(float f) {
    const uint32_t x = f32_bits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                 /* inf or nan */
        if (ax == 0x7f800000u) return sign | 0x7c00u;
        return sign | 0x7e00u | (uint16_t)((ax >> 13) & 0x1ffu);
    }
    if (ax >= 0x477ff000u) return sign | 0x7c00u;   /* rounds to >= 65520 -> inf */
    if (ax < 0x38800000u) {                  /* result is subnormal or zero: quantum 2^-24 */
        const float v = bits_f32(ax);
        /* v / 2^-24 is exact; rint gives round-half-even in the default rounding mode */
        const float q = rintf(v * 16777216.0f);
        return sign | (uint16_t)q;
    }
    const uint32_t mant = ax & 0x7fffffu;
    const uint32_t exp = (ax >> 23) - 112u;
    uint32_t h = (exp << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;   /* carries into the exponent as needed */
    return sign | (uint16_t)h;
}

/* ------------------------------------------------------------------ row sizes */

size_t oracle_row_size(int32_t type, int64_t n) {
    switch (type) {
        case ORACLE_T_F32:    return (size_t)n * 4;
        case ORACLE_T_F16:    return (size_t)n * 2;
        case ORACLE_T_Q5_0:   return (size_t)(n / 32) * 22;
        case ORACLE_T_Q8_0:   return (size_t)(n / 32) * 34;
        case ORACLE_T_Q4_K:   return (size_t)(n / 256) * 144;
        case ORACLE_T_Q8_K:   return (size_t)(n / 256) * 292;
        case ORACLE_T_IQ4_NL: return (size_t)(n / 32) * 18;
        case ORACLE_T_IQ2_S:  return (size_t)(n / 256) * 82;
        case ORACLE_T_IQ2_XXS: return (size_t)(n / 256) * 66;
        default:              return 0;
    }
}

int32_t oracle_vec_dot_type(int32_t wtype) {
    /* ggml-cpu/ggml-cpu.c type_traits_cpu: K-quants and IQ2_S pair with Q8_K, the 32-blocks with Q8_0 */
    switch (wtype) {
        case ORACLE_T_Q4_K: case ORACLE_T_IQ2_S: case ORACLE_T_IQ2_XXS: return ORACLE_T_Q8_K;
        case ORACLE_T_Q5_0: case ORACLE_T_IQ4_NL: return ORACLE_T_Q8_0;
        default: return wtype;
    }
}

/* ------------------------------------------------------------------ block field access
 * block_q4_K  (src/ggml-common.h:318): d f16 | dmin f16 | scales[12] | qs[128]          144 B / 256
 * block_iq2_s (ggml-common.h:385):     d f16 | qs[32] grid low bytes | signs[32] | qh[8] | scales[8]   82 B
 * block_q5_0  (ggml-common.h):         d f16 | qh[4] | qs[16]                            22 B / 32
 * block_iq4_nl (ggml-common.h):        d f16 | qs[16]                                    18 B / 32
 * block_q8_K  (ggml-common.h:361):     d f32 | qs[256] | bsums[16] i16                   292 B
 * block_q8_0:                          d f16 | qs[32]                                    34 B
 * block_iq2_xxs (ggml-common.h:371):   d f16 | 8 x (4 codebook indices u8 | 4 x 7-bit sign index
 *                                      + 4-bit sub-scale, one u32)                        66 B / 256
 */
static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* 6-bit sub-block scale and min of a Q4_K super-block (get_scale_min_k4, ggml-quants.c:822). */
static void q4k_scale_min(const uint8_t *sc, int j, int *s, int *m) {
    if (j < 4) {
        *s = sc[j] & 63;
        *m = sc[j + 4] & 63;
    } else {
        *s = (sc[j + 4] & 0x0f) | ((sc[j - 4] >> 6) << 4);
        *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

/* IQ2_S codebook index of 8-group g (0..31) of a super-block: low byte qs[g], two high bits from
 * qh[g/4] at bit 2*(g%4) (dequantize_row_iq2_s, ggml-quants.c:2471-2495). */
static int iq2s_index(const uint8_t *blk, int g) {
    const uint8_t *qs = blk + 2, *qh = blk + 66;
    return qs[g] | (((qh[g >> 2] >> (2 * (g & 3))) & 3) << 8);
}

/* ------------------------------------------------------------------ dequantisers */

void oracle_dequantize_row(int32_t type, const void *src, float *y, int64_t n) {
    const uint8_t *b = (const uint8_t *)src;
    if (type == ORACLE_T_Q4_K) {               /* dequantize_row_q4_K, ggml-quants.c:1471 */
        for (int64_t i = 0; i < n / 256; ++i, b += 144) {
            const float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
            const uint8_t *sc = b + 4, *q = b + 16;
            for (int c = 0; c < 4; ++c) {      /* 64 values per 32 bytes: low nibbles, then high */
                int s0, m0, s1, m1;
                q4k_scale_min(sc, 2 * c, &s0, &m0);
                q4k_scale_min(sc, 2 * c + 1, &s1, &m1);
                const float d0 = d * s0, o0 = dmin * m0, d1 = d * s1, o1 = dmin * m1;
                for (int l = 0; l < 32; ++l) y[l] = d0 * (q[l] & 0xf) - o0;
                for (int l = 0; l < 32; ++l) y[32 + l] = d1 * (q[l] >> 4) - o1;
                y += 64; q += 32;
            }
        }
    } else if (type == ORACLE_T_IQ2_S) {       /* dequantize_row_iq2_s, ggml-quants.c:2471 */
        for (int64_t i = 0; i < n / 256; ++i, b += 82) {
            const float d = h2f(rd16(b));
            const uint8_t *signs = b + 34, *scales = b + 74;
            for (int ib = 0; ib < 8; ++ib) {
                const float db0 = d * (0.5f + (scales[ib] & 0xf)) * 0.25f;
                const float db1 = d * (0.5f + (scales[ib] >> 4)) * 0.25f;
                for (int l = 0; l < 4; ++l) {
                    const int g = 4 * ib + l;
                    const uint64_t row = k_iq2s_grid[iq2s_index(b, g)];
                    const float dl = l < 2 ? db0 : db1;
                    for (int j = 0; j < 8; ++j) {
                        const float mag = (float)((row >> (8 * j)) & 0xff);
                        y[j] = dl * mag * ((signs[g] >> j) & 1 ? -1.f : 1.f);
                    }
                    y += 8;
                }
            }
        }
    } else if (type == ORACLE_T_IQ2_XXS) {     /* dequantize_row_iq2_xxs, ggml-quants.c:2416 */
        for (int64_t i = 0; i < n / 256; ++i, b += 66) {
            const float d = h2f(rd16(b));
            for (int ib = 0; ib < 8; ++ib) {
                const uint8_t *g8 = b + 2 + 8 * ib;
                const uint32_t hi = (uint32_t)g8[4] | ((uint32_t)g8[5] << 8) | ((uint32_t)g8[6] << 16) | ((uint32_t)g8[7] << 24);
                const float db = d * (0.5f + (float)(hi >> 28)) * 0.25f;
                for (int l = 0; l < 4; ++l) {
                    const uint64_t row = k_iq2xxs_grid[g8[l]];
                    const uint8_t sg = k_iq2xxs_signs[(hi >> (7 * l)) & 127];
                    for (int j = 0; j < 8; ++j)
                        y[j] = db * (float)((row >> (8 * j)) & 0xff) * ((sg >> j) & 1 ? -1.f : 1.f);
                    y += 8;
                }
            }
        }
    } else if (type == ORACLE_T_Q5_0) {        /* dequantize_row_q5_0, ggml-quants.c:442 */
        for (int64_t i = 0; i < n / 32; ++i, b += 22) {
            const float d = h2f(rd16(b));
            const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
            const uint8_t *qs = b + 6;
            for (int j = 0; j < 16; ++j) {
                const int v0 = (int)((qs[j] & 0xf) | (((qh >> j) & 1) << 4)) - 16;
                const int v1 = (int)((qs[j] >> 4) | (((qh >> (j + 16)) & 1) << 4)) - 16;
                y[j] = v0 * d;
                y[j + 16] = v1 * d;
            }
            y += 32;
        }
    } else if (type == ORACLE_T_IQ4_NL) {      /* dequantize_row_iq4_nl, ggml-quants.c:2653 */
        for (int64_t i = 0; i < n / 32; ++i, b += 18) {
            const float d = h2f(rd16(b));
            for (int j = 0; j < 16; ++j) {
                y[j] = d * k_iq4nl[b[2 + j] & 0xf];
                y[j + 16] = d * k_iq4nl[b[2 + j] >> 4];
            }
            y += 32;
        }
    } else if (type == ORACLE_T_Q8_0) {
        for (int64_t i = 0; i < n / 32; ++i, b += 34) {
            const float d = h2f(rd16(b));
            for (int j = 0; j < 32; ++j) y[j] = (int8_t)b[2 + j] * d;
            y += 32;
        }
    } else if (type == ORACLE_T_F32) {
        memcpy(y, src, (size_t)n * 4);
    }
}

/* ------------------------------------------------------------------ activation quantisers */

/* round-to-nearest-even through the 1.5*2^23 magic constant (nearest_int, ggml-quants.c:563) */
static int rne_int(float v) {
    const float t = v + 12582912.0f;
    return (int)(f32_bits(t) & 0x007fffffu) - 0x00400000;
}

/* Q8_K: quantize_row_q8_K on x86 is quantize_row_q8_K_ref (arch/x86/quants.c:505,
 * ggml-quants.c:2696): the scale comes from the signed value with the largest magnitude (first
 * one wins), iscale = -127/max, q = min(127, rne(iscale*x)), d = 1/iscale, bsums over 16s. */
static void quant_q8k(const float *x, uint8_t *y, int64_t n) {
    for (int64_t i = 0; i < n / 256; ++i, x += 256, y += 292) {
        float amax = 0.f, vmax = 0.f;
        for (int j = 0; j < 256; ++j) {
            const float a = fabsf(x[j]);
            if (a > amax) { amax = a; vmax = x[j]; }
        }
        int8_t *q = (int8_t *)(y + 4);
        int16_t bs[16];
        if (amax == 0.f) {
            memset(y, 0, 292);
            continue;
        }
        const float iscale = -127.f / vmax;
        for (int j = 0; j < 256; ++j) {
            const int v = rne_int(iscale * x[j]);
            q[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int l = 0; l < 16; ++l) s += q[16 * g + l];
            bs[g] = (int16_t)s;
        }
        const float d = 1.f / iscale;
        memcpy(y, &d, 4);
        memcpy(y + 260, bs, 32);
    }
}

/* Q8_0 with the AVX2 semantics of quantize_row_q8_0 (arch/x86/quants.c:302-350): d = amax/127
 * stored as f16, multiplier 127/amax (0 for an all-zero block), round-half-even. */
static void quant_q8_0(const float *x, uint8_t *y, int64_t n) {
    for (int64_t i = 0; i < n / 32; ++i, x += 32, y += 34) {
        float amax = 0.f;
        for (int j = 0; j < 32; ++j) { const float a = fabsf(x[j]); amax = a > amax ? a : amax; }
        const uint16_t dh = f2h(amax / 127.f);
        y[0] = (uint8_t)(dh & 0xff);
        y[1] = (uint8_t)(dh >> 8);
        const float id = amax != 0.f ? 127.f / amax : 0.f;
        for (int j = 0; j < 32; ++j) {
            const float r = rintf(x[j] * id);
            y[2 + j] = (uint8_t)(int8_t)(int)r;
        }
    }
}

void oracle_quantize_act(int32_t vdt, const float *x, void *y, int64_t n) {
    if (vdt == ORACLE_T_Q8_K) quant_q8k(x, (uint8_t *)y, n);
    else if (vdt == ORACLE_T_Q8_0) quant_q8_0(x, (uint8_t *)y, n);
}

/* ------------------------------------------------------------------ block dot products
 * The reference build runs the x86 AVX2 kernels of these dots (ggml-cpu/arch/x86/quants.c; the
 * AVX-512 VNNI and AVX-VNNI forms of the same kernels produce the same integer lanes). Their float
 * result depends on one fixed structure, restated here exactly:
 *   - 8 integer lanes per 32 values: lane L sums the 4 consecutive products at positions
 *     4L..4L+3 of every 32-value group (maddubs pairs, then madd_epi16 adding neighbouring pairs;
 *     the sub-block scales multiply inside the integer lanes);
 *   - per super-block (or 32-block) each lane converts to float and is fused-multiply-added into
 *     its own f32 accumulator with that block's scale (_mm256_fmadd_ps);
 *   - the 8 accumulators are reduced as hsum_float_8 (x86/quants.c:43-49):
 *     ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)).
 * Integer lane sums are exact (no int16 saturation is reachable with these formats), so every
 * rounding of the reference is reproduced and the dots are bit-equal to the reference's. */

static float hsum8(const float a[8]) {
    return ((a[0] + a[4]) + (a[2] + a[6])) + ((a[1] + a[5]) + (a[3] + a[7]));
}

/* ggml_vec_dot_q4_K_q8_K, AVX2 branch (x86/quants.c:1900-1982). Lane L of super-block i:
 * sum over the four 64-value chunks c of sc[2c] * sum_e q4lo[32c+4L+e] * q8[64c+4L+e] +
 * sc[2c+1] * sum_e q4hi[32c+4L+e] * q8[64c+32+4L+e]; d = y.d * x.d. The min term: four lanes
 * m = mins[2m] * q8s[2m] + mins[2m+1] * q8s[2m+1] with q8s[j] = bsums[2j] + bsums[2j+1] (the
 * 32-value sub-block sums), each fused into its own accumulator with dmin = -y.d * x.dmin, reduced
 * as (m0 + m2) + (m1 + m3) and added last. */
static float dot_q4k(int64_t n, const uint8_t *w, const uint8_t *x) {
    float acc[8] = {0}, accm[4] = {0};
    for (int64_t i = 0; i < n / 256; ++i, w += 144, x += 292) {
        float yd; memcpy(&yd, x, 4);
        const int8_t *q8 = (const int8_t *)(x + 4);
        int16_t bs[16]; memcpy(bs, x + 260, 32);
        const uint8_t *sc = w + 4, *q4 = w + 16;
        const float d = yd * h2f(rd16(w));
        const float dmin = -yd * h2f(rd16(w + 2));
        int scv[8], mnv[8];
        for (int j = 0; j < 8; ++j) q4k_scale_min(sc, j, &scv[j], &mnv[j]);
        for (int m = 0; m < 4; ++m) {
            const int prod = mnv[2 * m] * (bs[4 * m] + bs[4 * m + 1]) + mnv[2 * m + 1] * (bs[4 * m + 2] + bs[4 * m + 3]);
            accm[m] = fmaf(dmin, (float)prod, accm[m]);
        }
        for (int L = 0; L < 8; ++L) {
            int lane = 0;
            for (int c = 0; c < 4; ++c) {
                int lo = 0, hi = 0;
                for (int e = 0; e < 4; ++e) {
                    const int b = 32 * c + 4 * L + e;
                    lo += (q4[b] & 0xf) * q8[64 * c + 4 * L + e];
                    hi += (q4[b] >> 4) * q8[64 * c + 32 + 4 * L + e];
                }
                lane += scv[2 * c] * lo + scv[2 * c + 1] * hi;
            }
            acc[L] = fmaf(d, (float)lane, acc[L]);
        }
    }
    const float summ = (accm[0] + accm[2]) + (accm[1] + accm[3]);
    return hsum8(acc) + summ;
}

/* ggml_vec_dot_iq2_s_q8_K, AVX2 branch (x86/quants.c:2937-3025). Lane L of super-block i: sum over
 * the eight 32-blocks b of ls(b, half) * sum_e grid * sign * q8 at 32b+4L+e, where the half is the
 * block's first 16 values for L < 4 (low scale nibble) and its second 16 for L >= 4, ls = 2 * nibble
 * + 1; d = x.d * y.d; the total times 1/8. */
static float dot_iq2s(int64_t n, const uint8_t *w, const uint8_t *x) {
    float acc[8] = {0};
    for (int64_t i = 0; i < n / 256; ++i, w += 82, x += 292) {
        float yd; memcpy(&yd, x, 4);
        const int8_t *q8 = (const int8_t *)(x + 4);
        const uint8_t *signs = w + 34, *scales = w + 74;
        const float d = h2f(rd16(w)) * yd;
        int lane[8] = {0};
        for (int b = 0; b < 8; ++b) {
            for (int L = 0; L < 8; ++L) {
                int s = 0;
                for (int e = 0; e < 4; ++e) {
                    const int pos = 4 * L + e, g = 4 * b + pos / 8, j = pos % 8;
                    const int mag = (int)((k_iq2s_grid[iq2s_index(w, g)] >> (8 * j)) & 0xff);
                    const int v = (signs[g] >> j) & 1 ? -mag : mag;
                    s += v * q8[32 * b + pos];
                }
                const int ls = 2 * (L < 4 ? (scales[b] & 0xf) : (scales[b] >> 4)) + 1;
                lane[L] += ls * s;
            }
        }
        for (int L = 0; L < 8; ++L) acc[L] = fmaf(d, (float)lane[L], acc[L]);
    }
    return 0.125f * hsum8(acc);
}

/* ggml_vec_dot_q5_0_q8_0, AVX2 branch (x86/quants.c:1004-1043): values (q | qh bit << 4) - 16 in
 * element order; one accumulator, d = x.d * y.d per 32-block. */
static float dot_q5_0(int64_t n, const uint8_t *w, const uint8_t *x) {
    float acc[8] = {0};
    for (int64_t i = 0; i < n / 32; ++i, w += 22, x += 34) {
        const uint32_t qh = (uint32_t)w[2] | ((uint32_t)w[3] << 8) | ((uint32_t)w[4] << 16) | ((uint32_t)w[5] << 24);
        const int8_t *q8 = (const int8_t *)(x + 2);
        const float d = h2f(rd16(w)) * h2f(rd16(x));
        for (int L = 0; L < 8; ++L) {
            int s = 0;
            for (int e = 0; e < 4; ++e) {
                const int j = 4 * L + e;
                const int nib = j < 16 ? (w[6 + j] & 0xf) : (w[6 + j - 16] >> 4);
                s += ((int)(nib | (((qh >> j) & 1) << 4)) - 16) * q8[j];
            }
            acc[L] = fmaf(d, (float)s, acc[L]);
        }
    }
    return hsum8(acc);
}

/* ggml_vec_dot_iq4_nl_q8_0, AVX2 branch (x86/quants.c:3782-3815) and its scalar tail (:3854-3862):
 * even 32-blocks into one set of lane accumulators and odd blocks into another (d = y.d * x.d),
 * the two added lane by lane before the reduction; a last unpaired block is added in scalar. */
static float dot_iq4nl(int64_t n, const uint8_t *w, const uint8_t *x) {
    float acc[2][8] = {{0}};
    const int64_t nb = n / 32;
    int64_t ib = 0;
    for (; ib + 1 < nb; ib += 2) {
        for (int h = 0; h < 2; ++h) {
            const uint8_t *wb = w + (ib + h) * 18, *xb = x + (ib + h) * 34;
            const int8_t *q8 = (const int8_t *)(xb + 2);
            const float d = h2f(rd16(xb)) * h2f(rd16(wb));
            for (int L = 0; L < 8; ++L) {
                int s = 0;
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * L + e;
                    s += k_iq4nl[j < 16 ? (wb[2 + j] & 0xf) : (wb[2 + j - 16] >> 4)] * q8[j];
                }
                acc[h][L] = fmaf(d, (float)s, acc[h][L]);
            }
        }
    }
    float a[8];
    for (int L = 0; L < 8; ++L) a[L] = acc[0][L] + acc[1][L];
    float sumf = nb >= 2 ? hsum8(a) : 0.f;
    for (; ib < nb; ++ib) {
        const uint8_t *wb = w + ib * 18, *xb = x + ib * 34;
        const int8_t *q8 = (const int8_t *)(xb + 2);
        const float d = h2f(rd16(xb)) * h2f(rd16(wb));
        int s1 = 0, s2 = 0;
        for (int j = 0; j < 16; ++j) {
            s1 += q8[j] * k_iq4nl[wb[2 + j] & 0xf];
            s2 += q8[j + 16] * k_iq4nl[wb[2 + j] >> 4];
        }
        sumf += d * (float)(s1 + s2);
    }
    return sumf;
}

/* ggml_vec_dot_iq2_xxs_q8_K, AVX2 branch (x86/quants.c:2522-2563): lane L of super-block i sums,
 * over the eight 32-blocks b, (2 * ls_b + 1) * sum_e grid * sign * q8 at 32b+4L+e (the sign pattern
 * of each 8-group from the 7-bit index); d = x.d * y.d; the total times 1/8. */
static float dot_iq2xxs(int64_t n, const uint8_t *w, const uint8_t *x) {
    float acc[8] = {0};
    for (int64_t i = 0; i < n / 256; ++i, w += 66, x += 292) {
        float yd; memcpy(&yd, x, 4);
        const int8_t *q8 = (const int8_t *)(x + 4);
        const float d = h2f(rd16(w)) * yd;
        int lane[8] = {0};
        for (int b = 0; b < 8; ++b) {
            const uint8_t *g8 = w + 2 + 8 * b;
            const uint32_t hi = (uint32_t)g8[4] | ((uint32_t)g8[5] << 8) | ((uint32_t)g8[6] << 16) | ((uint32_t)g8[7] << 24);
            const int ls = (int)(2 * (hi >> 28) + 1);
            for (int L = 0; L < 8; ++L) {
                int s = 0;
                for (int e = 0; e < 4; ++e) {
                    const int pos = 4 * L + e, l = pos / 8, j = pos % 8;
                    const int mag = (int)((k_iq2xxs_grid[g8[l]] >> (8 * j)) & 0xff);
                    const uint8_t sg = k_iq2xxs_signs[(hi >> (7 * l)) & 127];
                    s += ((sg >> j) & 1 ? -mag : mag) * q8[32 * b + pos];
                }
                lane[L] += ls * s;
            }
        }
        for (int L = 0; L < 8; ++L) acc[L] = fmaf(d, (float)lane[L], acc[L]);
    }
    return 0.125f * hsum8(acc);
}

/* ggml_vec_dot_q8_0_q8_0, AVX2 branch (x86/quants.c:1170-1204): one accumulator, d = x.d * y.d */
static float dot_q8_0(int64_t n, const uint8_t *w, const uint8_t *x) {
    float acc[8] = {0};
    for (int64_t i = 0; i < n / 32; ++i, w += 34, x += 34) {
        const float d = h2f(rd16(w)) * h2f(rd16(x));
        for (int L = 0; L < 8; ++L) {
            int s = 0;
            for (int e = 0; e < 4; ++e) s += (int8_t)w[2 + 4 * L + e] * (int8_t)x[2 + 4 * L + e];
            acc[L] = fmaf(d, (float)s, acc[L]);
        }
    }
    return hsum8(acc);
}

float oracle_vec_dot(int32_t wtype, int64_t n, const void *w, const void *xq) {
    switch (wtype) {
        case ORACLE_T_IQ2_XXS: return dot_iq2xxs(n, (const uint8_t *)w, (const uint8_t *)xq);
        case ORACLE_T_Q8_0:   return dot_q8_0(n, (const uint8_t *)w, (const uint8_t *)xq);
        case ORACLE_T_Q4_K:   return dot_q4k(n, (const uint8_t *)w, (const uint8_t *)xq);
        case ORACLE_T_IQ2_S:  return dot_iq2s(n, (const uint8_t *)w, (const uint8_t *)xq);
        case ORACLE_T_Q5_0:   return dot_q5_0(n, (const uint8_t *)w, (const uint8_t *)xq);
        case ORACLE_T_IQ4_NL: return dot_iq4nl(n, (const uint8_t *)w, (const uint8_t *)xq);
        default:              return 0.f;
    }
}

/* ------------------------------------------------------------------ GeGLU */

/* tanh-form GELU as ggml-cpu evaluates it (ggml-cpu/vec.h:963-970), written in the same operation
 * order; with contraction off both sides round identically. */
static float gelu_tanh(float x) {
    const float c = 0.79788456080286535587989211986876f, a = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(c * x * (1.0f + a * x * x)));
}

uint16_t oracle_gelu_table(uint16_t h) { return f2h(gelu_tanh(h2f(h))); }   /* ggml-cpu.c:3792 */

static uint16_t *g_gelu_tab;

static const uint16_t *gelu_tab(void) {
    if (!g_gelu_tab) {
        uint16_t *t = (uint16_t *)malloc(sizeof(uint16_t) << 16);
        for (uint32_t h = 0; h < (1u << 16); ++h) t[h] = oracle_gelu_table((uint16_t)h);
        g_gelu_tab = t;
    }
    return g_gelu_tab;
}

/* ggml_vec_geglu_f32 with GGML_GELU_FP16 (ggml-cpu/vec.h:1414-1430) */
void oracle_geglu(int64_t n, float *y, const float *gate, const float *up) {
    const uint16_t *t = gelu_tab();
    for (int64_t i = 0; i < n; ++i) {
        const float g = gate[i];
        if (g <= -10.0f) y[i] = 0.0f;
        else if (g >= 10.0f) y[i] = g * up[i];
        else y[i] = h2f(t[f2h(g)]) * up[i];
    }
}

/* ------------------------------------------------------------------ routing */

/* k largest values, ordered by (value desc, index asc); the reference's argsort is an unstable
 * std::sort (ggml-cpu/ops.cpp:8211-8255), so exact ties are resolved here to the lowest index. */
void oracle_topk(const float *v, int32_t n, int32_t k, int32_t *ids) {
    for (int j = 0; j < k; ++j) {
        int best = -1;
        for (int e = 0; e < n; ++e) {
            int taken = 0;
            for (int i = 0; i < j; ++i) if (ids[i] == e) { taken = 1; break; }
            if (taken) continue;
            if (best < 0 || v[e] > v[best]) best = e;
        }
        ids[j] = best;
    }
}

static int pair_hot(const oracle_layer *L, int e, int *slot) {
    if (L->n_slots <= 0 || !L->exp_slot) return 0;
    const int s = L->exp_slot[e];
    if (s >= 0 && s < L->n_slots && L->slot_state[s] == 2 && L->slot_exp[s] == e) { *slot = s; return 1; }
    return 0;
}

int oracle_moe_layer(const oracle_layer *L, oracle_layer_out *o) {
    const int d = L->d_model, E = L->n_expert, k = L->top_k, T = L->n_tokens, nff = L->n_ff;
    float *logit = (float *)malloc(sizeof(float) * E), *prob = (float *)malloc(sizeof(float) * E);
    float *h = (float *)malloc(sizeof(float) * 2 * nff), *a = (float *)malloc(sizeof(float) * nff);
    float *y = (float *)malloc(sizeof(float) * d);
    float *acc = (float *)malloc(sizeof(float) * d);
    int32_t *ids = (int32_t *)malloc(sizeof(int32_t) * k);
    float *w = (float *)malloc(sizeof(float) * k);
    uint8_t *xq = (uint8_t *)malloc(oracle_row_size(ORACLE_T_Q8_K, d) + oracle_row_size(ORACLE_T_Q8_0, d));
    uint8_t *aq = (uint8_t *)malloc(oracle_row_size(ORACLE_T_Q8_0, nff) + oracle_row_size(ORACLE_T_Q8_K, nff + 256));

    for (int t = 0; t < T; ++t) {
        const float *xt = L->x + (size_t)t * d;
        const float *xr = L->x_router ? L->x_router + (size_t)t * d : xt;
        /* router logits (mul_mat f32; summed in double here) + optional bias (llama-graph.cpp:1530-1540) */
        for (int e = 0; e < E; ++e) {
            double s = 0.0;
            const float *wr = L->w_router + (size_t)e * d;
            for (int i = 0; i < d; ++i) s += (double)wr[i] * (double)xr[i];
            logit[e] = (float)s;
            if (L->b_router) logit[e] += L->b_router[e];
        }
        /* softmax (ggml-cpu/ops.cpp:5427-5443): max, exp(l - max), double sum, scale by 1/sum */
        float mx = -INFINITY;
        for (int e = 0; e < E; ++e) mx = logit[e] > mx ? logit[e] : mx;
        double sum = 0.0;
        for (int e = 0; e < E; ++e) { prob[e] = expf(logit[e] - mx); sum += prob[e]; }
        const float inv = (float)(1.0 / sum);
        for (int e = 0; e < E; ++e) prob[e] *= inv;
        if (L->ids_in) memcpy(ids, L->ids_in + (size_t)t * k, sizeof(int32_t) * k);
        else oracle_topk(prob, E, k, ids);
        /* weights: get_rows, sum_rows (double), clamp, div (llama-graph.cpp:1626-1648) */
        double ws = 0.0;
        for (int j = 0; j < k; ++j) { w[j] = prob[ids[j]]; ws += w[j]; }
        float wsf = (float)ws;
        if (wsf < 6.103515625e-5f) wsf = 6.103515625e-5f;
        for (int j = 0; j < k; ++j) w[j] = w[j] / wsf;

        if (o->logits) memcpy(o->logits + (size_t)t * E, logit, sizeof(float) * E);
        if (o->probs) memcpy(o->probs + (size_t)t * E, prob, sizeof(float) * E);
        if (o->ids) memcpy(o->ids + (size_t)t * k, ids, sizeof(int32_t) * k);
        if (o->weights) memcpy(o->weights + (size_t)t * k, w, sizeof(float) * k);

        for (int j = 0; j < k; ++j) {
            const int e = ids[j], p = t * k + j;
            int slot = -1;
            const int hot = pair_hot(L, e, &slot);
            const int tgu = hot ? L->hot_type_gu : L->cold_type_gu;
            const int tdn = hot ? L->hot_type_down : L->cold_type_down;
            const uint8_t *wgu = (const uint8_t *)(hot ? L->hot_gu : L->cold_gu);
            const uint8_t *wdn = (const uint8_t *)(hot ? L->hot_down : L->cold_down);
            const int widx = hot ? slot : e;
            const size_t rgu = oracle_row_size(tgu, d), rdn = oracle_row_size(tdn, nff);
            wgu += (size_t)widx * 2 * nff * rgu;
            wdn += (size_t)widx * d * rdn;
            /* gate_up: x quantised to the weight type's vec_dot_type (ggml-cpu.c:1581-1610) */
            if (L->gate_up_in) {
                memcpy(h, L->gate_up_in + (size_t)p * 2 * nff, sizeof(float) * 2 * nff);
            } else {
                oracle_quantize_act(oracle_vec_dot_type(tgu), xt, xq, d);
                for (int r = 0; r < 2 * nff; ++r) h[r] = oracle_vec_dot(tgu, d, wgu + (size_t)r * rgu, xq);
            }
            if (L->gelu_tanh) {
                for (int i = 0; i < nff; ++i) a[i] = gelu_tanh(h[i]) * h[nff + i];
            } else {
                oracle_geglu(nff, a, h, h + nff);
            }
            oracle_quantize_act(oracle_vec_dot_type(tdn), a, aq, nff);
            const float sc = hot ? (L->s_hot ? L->s_hot[slot] : 1.f) : (L->s_cold ? L->s_cold[e] : 1.f);
            for (int r = 0; r < d; ++r) {
                y[r] = oracle_vec_dot(tdn, nff, wdn + (size_t)r * rdn, aq);
                if (hot ? L->s_hot != NULL : L->s_cold != NULL) y[r] = y[r] * sc;
            }
            if (o->gate_up) memcpy(o->gate_up + (size_t)p * 2 * nff, h, sizeof(float) * 2 * nff);
            if (o->act) memcpy(o->act + (size_t)p * nff, a, sizeof(float) * nff);
            if (o->down) memcpy(o->down + (size_t)p * d, y, sizeof(float) * d);
            /* weighting then the j-ordered add chain (llama-graph.cpp:1814-1848) */
            for (int r = 0; r < d; ++r) {
                const float v = y[r] * w[j];
                acc[r] = j == 0 ? v : acc[r] + v;
            }
        }
        memcpy(o->out + (size_t)t * d, acc, sizeof(float) * d);
    }
    free(logit); free(prob); free(h); free(a); free(y); free(acc); free(ids); free(w); free(xq); free(aq);
    return 1;
}

/* ggml_rms_norm, row by row (ggml-cpu/ops.cpp:3808-3838, ggml_compute_forward_rms_norm_f32): sum
 * of x*x (each product in float) accumulated in double, mean = sum / n, scale = 1.0f / sqrtf(mean +
 * eps), y = x * scale; then the ggml_scale node (ops.cpp:4522-4529: y * s) and the ggml_mul node
 * with a broadcast [n] weight (y * w[i]) when the caller's graph has them */
void oracle_rms_norm(const float *x, const float *w, float s, float *y, int64_t rows, int64_t n, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; ++i) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / (double)n);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < n; ++i) {
            float v = xr[i] * scale;
            if (s != 1.0f) v = v * s;
            if (w) v = v * w[i];
            y[r * n + i] = v;
        }
    }
}
