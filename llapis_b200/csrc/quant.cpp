// Host-side expert-weight quantiser (moeb_quantize_weights): the ggml formats the MoE path serves,
// restated from the reference quantiser without an importance matrix (IQ2_XXS, which ggml
// quantises only with one, with a uniform one) (ggml_quantize_chunk, ggml/src/ggml.c:7761):
//   Q4_K   quantize_row_q4_K_ref + make_qkx2_quants  (ggml-quants.c:1399, :741)
//   Q5_0   quantize_row_q5_0_ref                      (ggml-quants.c:149)
//   IQ4_NL quantize_row_iq4_nl_impl, 7 scale trials    (ggml-quants.c:4894, :5005)
//   IQ2_S  quantize_row_iq2_s_impl + the codebook map  (ggml-quants.c:5070, :2781, :3198)
//   IQ2_XXS quantize_row_iq2_xxs_impl + make_qp_quants (ggml-quants.c:3222, :1018)
//   Q8_0   quantize_row_q8_0_ref                      (ggml-quants.c:238)
// Every float expression keeps the reference's evaluation order and this file is compiled with
// -ffp-contract=off, so the output bytes equal the reference quantiser's (checked by the tests).
// Rows are independent and are spread over host threads.
#include "moeb200.h"
#include "params.h"

#include <immintrin.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "ggml_tables.inc"

using namespace moeb;

namespace {

inline uint16_t to_f16(float f) { return _cvtss_sh(f, 0); }
inline float from_f16(uint16_t h) { return _cvtsh_ss(h); }

// round-to-nearest-even through the 1.5 * 2^23 constant (valid for |v| < 2^22)
inline int rne(float v) {
    const float t = v + 12582912.0f;
    int32_t i;
    memcpy(&i, &t, 4);
    return (i & 0x007fffff) - 0x00400000;
}

// ---------------------------------------------------------------- Q5_0
void q5_0_row(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / 32; ++b, x += 32, y += B_Q5_0) {
        float amax = 0.f, vmax = 0.f;
        for (int j = 0; j < 32; ++j)
            if (amax < fabsf(x[j])) { amax = fabsf(x[j]); vmax = x[j]; }
        const float d = vmax / -16;
        const float id = d ? 1.0f / d : 0.0f;
        const uint16_t dh = to_f16(d);
        memcpy(y, &dh, 2);
        uint32_t qh = 0;
        for (int j = 0; j < 16; ++j) {
            const float x0 = x[j] * id, x1 = x[16 + j] * id;
            const uint8_t v0 = (uint8_t)std::min(31, (int)(int8_t)(x0 + 16.5f));
            const uint8_t v1 = (uint8_t)std::min(31, (int)(int8_t)(x1 + 16.5f));
            y[6 + j] = (uint8_t)((v0 & 0x0f) | ((v1 & 0x0f) << 4));
            qh |= (uint32_t)((v0 & 0x10u) >> 4) << j;
            qh |= (uint32_t)((v1 & 0x10u) >> 4) << (j + 16);
        }
        memcpy(y + 2, &qh, 4);
    }
}

// ---------------------------------------------------------------- Q4_K
// scale/min search for one 32-value sub-block with the asymmetric model x ~ scale*L + min
float qkx2_search(const float *x, const float *w, uint8_t *L, float *neg_min, uint8_t *Laux) {
    const int n = 32, nmax = 15, nstep = 20;
    const float rmin = -1.f, rdelta = 0.1f;
    float mn = x[0], mx = x[0];
    float sum_w = w[0];
    float sum_x = sum_w * x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
        const float wi = w[i];
        sum_w += wi;
        sum_x += wi * x[i];
    }
    if (mn > 0) mn = 0;
    if (mx == mn) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        *neg_min = -mn;
        return 0.f;
    }
    float iscale = nmax / (mx - mn);
    float scale = 1 / iscale;
    float best = 0;
    for (int i = 0; i < n; ++i) {
        const int l = rne(iscale * (x[i] - mn));
        L[i] = (uint8_t)std::max(0, std::min(nmax, l));
        float diff = scale * L[i] + mn - x[i];
        diff = diff * diff;
        best += w[i] * diff;
    }
    for (int is = 0; is <= nstep; ++is) {
        iscale = (rmin + rdelta * is + nmax) / (mx - mn);
        float sl = 0, sl2 = 0, sxl = 0;
        for (int i = 0; i < n; ++i) {
            int l = rne(iscale * (x[i] - mn));
            l = std::max(0, std::min(nmax, l));
            Laux[i] = (uint8_t)l;
            const float wi = w[i];
            sl += wi * l;
            sl2 += wi * l * l;
            sxl += wi * l * x[i];
        }
        const float D = sum_w * sl2 - sl * sl;
        if (D > 0) {
            float s = (sum_w * sxl - sum_x * sl) / D;
            float m = (sl2 * sum_x - sl * sxl) / D;
            if (m > 0) {
                m = 0;
                s = sxl / sl2;
            }
            float err = 0;
            for (int i = 0; i < n; ++i) {
                float diff = s * Laux[i] + m - x[i];
                diff = diff * diff;
                err += w[i] * diff;
            }
            if (err < best) {
                for (int i = 0; i < n; ++i) L[i] = Laux[i];
                best = err;
                scale = s;
                mn = m;
            }
        }
    }
    *neg_min = -mn;
    return scale;
}

void q4k_get_scale_min(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j - 0] >> 6) << 4);
    }
}

void q4_k_row(const float *x, uint8_t *y, int64_t n) {
    uint8_t L[256], Laux[32];
    float w[32], mins[8], scales[8];
    for (int64_t b = 0; b < n / 256; ++b, x += 256, y += B_Q4_K) {
        memset(y, 0, B_Q4_K);
        uint8_t *sc = y + 4;
        float max_scale = 0, max_min = 0;
        for (int j = 0; j < 8; ++j) {
            float sum_x2 = 0;
            for (int l = 0; l < 32; ++l) sum_x2 += x[32 * j + l] * x[32 * j + l];
            const float av_x = sqrtf(sum_x2 / 32);
            for (int l = 0; l < 32; ++l) w[l] = av_x + fabsf(x[32 * j + l]);
            scales[j] = qkx2_search(x + 32 * j, w, L + 32 * j, &mins[j], Laux);
            if (scales[j] > max_scale) max_scale = scales[j];
            if (mins[j] > max_min) max_min = mins[j];
        }
        const float inv_scale = max_scale > 0 ? 63.f / max_scale : 0.f;
        const float inv_min = max_min > 0 ? 63.f / max_min : 0.f;
        for (int j = 0; j < 8; ++j) {
            uint8_t ls = (uint8_t)rne(inv_scale * scales[j]);
            uint8_t lm = (uint8_t)rne(inv_min * mins[j]);
            ls = std::min<uint8_t>(63, ls);
            lm = std::min<uint8_t>(63, lm);
            if (j < 4) {
                sc[j] = ls;
                sc[j + 4] = lm;
            } else {
                sc[j + 4] = (uint8_t)((ls & 0xF) | ((lm & 0xF) << 4));
                sc[j - 4] |= (uint8_t)((ls >> 4) << 6);
                sc[j - 0] |= (uint8_t)((lm >> 4) << 6);
            }
        }
        const uint16_t dh = to_f16(max_scale / 63.f), mh = to_f16(max_min / 63.f);
        memcpy(y, &dh, 2);
        memcpy(y + 2, &mh, 2);
        for (int j = 0; j < 8; ++j) {
            uint8_t s, m;
            q4k_get_scale_min(j, sc, &s, &m);
            const float d = from_f16(dh) * s;
            if (!d) continue;
            const float dm = from_f16(mh) * m;
            for (int ii = 0; ii < 32; ++ii) {
                const int l = rne((x[32 * j + ii] + dm) / d);
                L[32 * j + ii] = (uint8_t)std::max(0, std::min(15, l));
            }
        }
        uint8_t *q = y + 16;
        for (int j = 0; j < 256; j += 64) {
            for (int l = 0; l < 32; ++l) q[l] = (uint8_t)(L[j + l] | (L[j + l + 32] << 4));
            q += 32;
        }
    }
}

// ---------------------------------------------------------------- IQ4_NL
const int8_t kIq4nl[16] = MOE_IQ4NL_VALUES_INIT;

int nearest_level(float x) {
    const int8_t *v = kIq4nl;
    if (x <= v[0]) return 0;
    if (x >= v[15]) return 15;
    int lo = 0, hi = 15;
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (x < v[mid]) hi = mid; else lo = mid;
    }
    return x - v[hi - 1] < v[hi] - x ? hi - 1 : hi;
}

void iq4_nl_row(const float *x, uint8_t *y, int64_t n) {
    const int8_t *vals = kIq4nl;
    const int ntry = 7;
    for (int64_t b = 0; b < n / 32; ++b, x += 32, y += B_IQ4_NL) {
        float w[32];
        uint8_t L[32];
        memset(y + 2, 0, 16);
        for (int j = 0; j < 32; ++j) w[j] = x[j] * x[j];
        float amax = 0, vmax = 0;
        for (int j = 0; j < 32; ++j) {
            const float ax = fabsf(x[j]);
            if (ax > amax) { amax = ax; vmax = x[j]; }
        }
        float scale = 0;
        if (!(amax < 1e-15f)) {
            float d = -vmax / vals[0];
            float id = 1 / d;
            float sqx = 0, sq2 = 0;
            for (int j = 0; j < 32; ++j) {
                const float al = id * x[j];
                const int l = nearest_level(al);
                L[j] = (uint8_t)l;
                const float q = vals[l];
                const float wj = w[j];
                sqx += wj * q * x[j];
                sq2 += wj * q * q;
            }
            d = sq2 > 0 ? sqx / sq2 : 0.f;
            float best = d * sqx;
            for (int itry = -ntry; itry <= ntry; ++itry) {
                id = (itry + vals[0]) / vmax;
                sqx = sq2 = 0;
                for (int j = 0; j < 32; ++j) {
                    const float al = id * x[j];
                    const int l = nearest_level(al);
                    const float q = vals[l];
                    const float wj = w[j];
                    sqx += wj * q * x[j];
                    sq2 += wj * q * q;
                }
                if (sq2 > 0 && sqx * sqx > best * sq2) {
                    d = sqx / sq2;
                    best = d * sqx;
                }
            }
            scale = d;
        }
        const uint16_t dh = to_f16(scale);
        memcpy(y, &dh, 2);
        const float id = scale ? 1 / scale : 0;
        for (int j = 0; j < 32; ++j) L[j] = (uint8_t)nearest_level(id * x[j]);
        for (int j = 0; j < 16; ++j) y[2 + j] = (uint8_t)(L[j] | (L[16 + j] << 4));
    }
}

// ---------------------------------------------------------------- IQ2_S / IQ2_XXS codebook search
// The quantisers work on a codebook in its search form: each row is 8 levels l in {0,1,2} (value
// 2l+1), packed as u = sum l_i << 2i. `map[u]` is the codebook row of u, or -(offset+1) into `nbr`
// where the rows at the `nwant` smallest squared distances from u are listed (count first, then
// rows in (distance, row) order) — the layout of iq2xs_init_impl (ggml-quants.c:2781-3190; nwant
// is 1 for IQ2_S and 2 for IQ2_XXS).
struct Iq2sSearch {
    std::vector<uint64_t> grid;   // rows as int8 levels 1/3/5
    std::vector<int> map;         // 43692 entries
    std::vector<uint16_t> nbr;
};

// dq: the dequantisation rows (magnitudes 8, 25, 43 per byte)
void build_search(Iq2sSearch &S, const uint64_t *dq, int rows, int nwant) {
    S.grid.resize(rows);
    for (int r = 0; r < rows; ++r) {
        uint64_t g = 0;
        for (int i = 0; i < 8; ++i) {
            const int mag = (int)((dq[r] >> (8 * i)) & 0xff);
            const int l = mag == 8 ? 0 : mag == 25 ? 1 : 2;
            g |= (uint64_t)(2 * l + 1) << (8 * i);
        }
        S.grid[r] = g;
    }
    const int kmap = 43692;
    S.map.assign(kmap, -1);
    for (int r = 0; r < rows; ++r) {
        int u = 0;
        for (int i = 0; i < 8; ++i) u |= ((int)(((S.grid[r] >> (8 * i)) & 0xff) - 1) / 2) << (2 * i);
        S.map[u] = r;
    }
    std::vector<std::pair<int, int>> dist(rows);
    for (int u = 0; u < kmap; ++u) {
        if (S.map[u] >= 0) continue;
        int pos[8];
        for (int i = 0; i < 8; ++i) pos[i] = 2 * ((u >> (2 * i)) & 3) + 1;
        for (int r = 0; r < rows; ++r) {
            int d2 = 0;
            for (int i = 0; i < 8; ++i) {
                const int q = (int)((S.grid[r] >> (8 * i)) & 0xff) - pos[i];
                d2 += q * q;
            }
            dist[r] = {d2, r};
        }
        std::sort(dist.begin(), dist.end());
        S.map[u] = -((int)S.nbr.size() + 1);
        const size_t at = S.nbr.size();
        S.nbr.push_back(0);
        int n = 0, have = 1, d2 = dist[0].first;
        for (int r = 0; r < rows; ++r) {
            if (dist[r].first > d2) {   // the next distinct distance
                if (have == nwant) break;
                d2 = dist[r].first;
                ++have;
            }
            S.nbr.push_back((uint16_t)dist[r].second);
            ++n;
        }
        S.nbr[at] = (uint16_t)n;
    }
}

const Iq2sSearch &iq2s_search() {
    static Iq2sSearch S;
    static std::once_flag once;
    std::call_once(once, [] {
        static const uint64_t dq[1024] = MOE_IQ2S_GRID_INIT;
        build_search(S, dq, 1024, 1);
    });
    return S;
}

const Iq2sSearch &iq2xxs_search() {
    static Iq2sSearch S;
    static std::once_flag once;
    std::call_once(once, [] {
        static const uint64_t dq[256] = MOE_IQ2XXS_GRID_INIT;
        build_search(S, dq, 256, 2);
    });
    return S;
}

int best_neighbour(const Iq2sSearch &S, const uint16_t *list, const float *xval, const float *w, float scale, int8_t *L) {
    const int n = list[0];
    float best = FLT_MAX;
    int row = -1;
    for (int j = 1; j <= n; ++j) {
        const uint64_t g = S.grid[list[j]];
        float d2 = 0;
        for (int i = 0; i < 8; ++i) {
            const float q = (float)(int8_t)((g >> (8 * i)) & 0xff);
            const float diff = scale * q - xval[i];
            d2 += w[i] * diff * diff;
        }
        if (d2 < best) { best = d2; row = list[j]; }
    }
    const uint64_t g = S.grid[row];
    for (int i = 0; i < 8; ++i) L[i] = (int8_t)(((int)((g >> (8 * i)) & 0xff) - 1) / 2);
    return row;
}

void iq2_s_row(const float *x, uint8_t *y, int64_t n) {
    const Iq2sSearch &S = iq2s_search();
    const int kMaxQ = 3;
    for (int64_t b = 0; b < n / 256; ++b, x += 256, y += B_IQ2_S) {
        memset(y, 0, B_IQ2_S);
        uint8_t *qs = y + 2, *signs = y + 34, *qh = y + 66, *scl = y + 74;
        float scales[16], weight[16], xval[16], waux[16];
        int8_t L[16], Laux[16];
        bool on_grid[2], on_grid_aux[2];
        uint8_t bsign[2];
        float max_scale = 0;
        float sumx2 = 0;
        for (int i = 0; i < 256; ++i) sumx2 += x[i] * x[i];
        const float sigma2 = 2 * sumx2 / 256;
        for (int ib = 0; ib < 16; ++ib) {
            const float *xb = x + 16 * ib;
            for (int i = 0; i < 16; ++i) weight[i] = 0.25f * sigma2 + xb[i] * xb[i];
            for (int i = 0; i < 16; ++i) waux[i] = sqrtf(weight[i]);
            for (int k = 0; k < 2; ++k) {
                uint8_t s = 0;
                for (int i = 0; i < 8; ++i) {
                    if (xb[8 * k + i] >= 0) xval[8 * k + i] = xb[8 * k + i];
                    else { xval[8 * k + i] = -xb[8 * k + i]; s |= (uint8_t)(1 << i); }
                }
                bsign[k] = s;
            }
            float mx = xval[0];
            for (int i = 1; i < 16; ++i) mx = std::max(mx, xval[i]);
            memset(L, 0, 16);
            if (mx < 1e-8f) {
                scales[ib] = 0;
                continue;
            }
            float best = 0;
            float scale = mx / (2 * kMaxQ - 1);
            on_grid[0] = on_grid[1] = true;
            for (int is = -9; is <= 9; ++is) {
                const float id = (2 * kMaxQ - 1 + is * 0.1f) / mx;
                const float this_scale = 1 / id;
                for (int k = 0; k < 2; ++k) {
                    for (int i = 0; i < 8; ++i) {
                        const int l = rne(0.5f * (id * xval[8 * k + i] - 1));
                        Laux[8 * k + i] = (int8_t)std::max(0, std::min(kMaxQ - 1, l));
                    }
                    int u = 0;
                    for (int i = 0; i < 8; ++i) u |= Laux[8 * k + i] << (2 * i);
                    on_grid_aux[k] = true;
                    if (S.map[u] < 0) {
                        on_grid_aux[k] = false;
                        best_neighbour(S, S.nbr.data() - S.map[u] - 1, xval + 8 * k, waux + 8 * k, this_scale, Laux + 8 * k);
                    }
                }
                float sqx = 0, sq2 = 0;
                for (int i = 0; i < 16; ++i) {
                    const float w = weight[i];
                    const float q = 2 * Laux[i] + 1;
                    sqx += w * xval[i] * q;
                    sq2 += w * q * q;
                }
                if (sq2 > 0 && sqx * sqx > best * sq2) {
                    scale = sqx / sq2;
                    best = scale * sqx;
                    for (int i = 0; i < 16; ++i) L[i] = Laux[i];
                    for (int k = 0; k < 2; ++k) on_grid[k] = on_grid_aux[k];
                }
            }
            int off_grid = 0;
            for (int k = 0; k < 2; ++k) if (!on_grid[k]) ++off_grid;
            if (off_grid > 0 && scale > 0) {
                const float id = 1 / scale;
                for (int k = 0; k < 2; ++k) {
                    if (on_grid[k]) continue;
                    int u = 0;
                    for (int i = 0; i < 8; ++i) {
                        int l = rne(0.5f * (id * xval[8 * k + i] - 1));
                        l = std::max(0, std::min(kMaxQ - 1, l));
                        u |= l << (2 * i);
                        L[8 * k + i] = (int8_t)l;
                    }
                    if (S.map[u] < 0)
                        best_neighbour(S, S.nbr.data() - S.map[u] - 1, xval + 8 * k, waux + 8 * k, scale, L + 8 * k);
                }
                float sqx = 0, sq2 = 0;
                for (int i = 0; i < 16; ++i) {
                    const float w = weight[i];
                    const float q = 2 * L[i] + 1;
                    sqx += w * xval[i] * q;
                    sq2 += w * q * q;
                }
                if (sq2 > 0) scale = sqx / sq2;
            }
            if (scale < 0) {
                scale = -scale;
                for (int k = 0; k < 2; ++k) bsign[k] = (uint8_t)~bsign[k];
            }
            for (int k = 0; k < 2; ++k) {
                int u = 0;
                for (int i = 0; i < 8; ++i) u |= L[8 * k + i] << (2 * i);
                const int row = S.map[u];   // on the codebook by construction
                const int i8 = 2 * ib + k;
                qs[i8] = (uint8_t)(row & 255);
                qh[i8 / 4] |= (uint8_t)((row >> 8) << (2 * (i8 % 4)));
                signs[i8] = bsign[k];
            }
            scales[ib] = scale;
            max_scale = std::max(max_scale, scale);
        }
        if (!max_scale) continue;
        const float d = max_scale / 31;
        const uint16_t dh = to_f16(d * 0.9875f);
        memcpy(y, &dh, 2);
        const float id = 1 / d;
        for (int ib = 0; ib < 16; ++ib) {
            int l = rne(0.5f * (id * scales[ib] - 1));
            l = std::max(0, std::min(15, l));
            if (ib % 2 == 0) scl[ib / 2] = (uint8_t)l;
            else scl[ib / 2] |= (uint8_t)(l << 4);
        }
    }
}

// Q8_0 weights (quantize_row_q8_0_ref, ggml-quants.c:238-261): d = amax / 127, q = roundf(x / d)
// (half away from zero)
void q8_0_row(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / 32; ++b, x += 32, y += B_Q8_0) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, fabsf(x[j]));
        const float d = amax / 127;
        const float id = d ? 1.0f / d : 0.0f;
        const uint16_t dh = to_f16(d);
        memcpy(y, &dh, 2);
        for (int j = 0; j < 32; ++j) y[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
    }
}

// make_qp_quants (ggml-quants.c:1018-1089): levels 0..nmax for non-negative x with weights w,
// a scale search over nine candidates, then up to five rounds of single-level improvements
float make_qp_quants(int n, int nmax, const float *x, uint8_t *L, const float *w) {
    float max = 0;
    for (int i = 0; i < n; ++i) max = std::max(max, x[i]);
    if (max < 1e-15f) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        return 0.f;
    }
    float iscale = nmax / max;
    for (int i = 0; i < n; ++i) L[i] = (uint8_t)rne(iscale * x[i]);
    const float scale = 1 / iscale;
    float best_mse = 0;
    for (int i = 0; i < n; ++i) {
        const float diff = x[i] - scale * L[i];
        best_mse += w[i] * diff * diff;
    }
    for (int is = -4; is <= 4; ++is) {
        if (is == 0) continue;
        const float iscale_is = (0.1f * is + nmax) / max;
        const float scale_is = 1 / iscale_is;
        float mse = 0;
        for (int i = 0; i < n; ++i) {
            const int l = std::min(nmax, rne(iscale_is * x[i]));
            const float diff = x[i] - scale_is * l;
            mse += w[i] * diff * diff;
        }
        if (mse < best_mse) {
            best_mse = mse;
            iscale = iscale_is;
        }
    }
    float sumlx = 0, suml2 = 0;
    for (int i = 0; i < n; ++i) {
        const int l = std::min(nmax, rne(iscale * x[i]));
        L[i] = (uint8_t)l;
        sumlx += w[i] * x[i] * l;
        suml2 += w[i] * l * l;
    }
    for (int itry = 0; itry < 5; ++itry) {
        int changed = 0;
        for (int i = 0; i < n; ++i) {
            float slx = sumlx - w[i] * x[i] * L[i];
            float sl2 = suml2 - w[i] * L[i] * L[i];
            if (slx > 0 && sl2 > 0) {
                const int nl = std::min(nmax, rne(x[i] * sl2 / slx));
                if (nl != L[i]) {
                    slx += w[i] * x[i] * nl;
                    sl2 += w[i] * nl * nl;
                    if (slx * slx * suml2 > sumlx * sumlx * sl2) {
                        L[i] = (uint8_t)nl;
                        sumlx = slx;
                        suml2 = sl2;
                        ++changed;
                    }
                }
            }
        }
        if (!changed) break;
    }
    return suml2 > 0.0f ? sumlx / suml2 : 0.0f;
}

// IQ2_XXS (quantize_row_iq2_xxs_impl, ggml-quants.c:3222-3397) with a uniform importance matrix
// (the reference quantises this type only with one): per 32-block a weighted fit of four codebook
// rows and one scale, each 8-group's signs made even in number (the cheapest value flipped), the
// scales coded in 4 bits against max_scale / 31.
void iq2_xxs_row(const float *x, uint8_t *y, int64_t n) {
    const Iq2sSearch &S = iq2xxs_search();
    const int kMaxQ = 3;
    for (int64_t b = 0; b < n / 256; ++b, x += 256, y += B_IQ2_XXS) {
        uint32_t q2[16] = {};
        float scales[8], weight[32], xval[32], waux[32];
        int8_t L[32], Laux[32];
        uint8_t block_signs[4];
        float max_scale = 0;
        float sumx2 = 0;
        for (int i = 0; i < 256; ++i) sumx2 += x[i] * x[i];
        const float sigma2 = sumx2 / 256;
        for (int ib = 0; ib < 8; ++ib) {
            const float *xb = x + 32 * ib;
            for (int i = 0; i < 32; ++i) weight[i] = 1.0f * sqrtf(sigma2 + xb[i] * xb[i]);
            for (int i = 0; i < 32; ++i) waux[i] = sqrtf(weight[i]);
            for (int k = 0; k < 4; ++k) {
                int nflip = 0;
                uint8_t sg = 0;
                for (int i = 0; i < 8; ++i) {
                    if (xb[8 * k + i] >= 0) xval[8 * k + i] = xb[8 * k + i];
                    else { xval[8 * k + i] = -xb[8 * k + i]; ++nflip; sg |= (uint8_t)(1 << i); }
                }
                if (nflip % 2) {
                    int imin = 0;
                    float mn = weight[8 * k] * xb[8 * k] * xb[8 * k];
                    for (int i = 1; i < 8; ++i) {
                        const float ax = weight[8 * k + i] * xb[8 * k + i] * xb[8 * k + i];
                        if (ax < mn) { mn = ax; imin = i; }
                    }
                    xval[8 * k + imin] = -xval[8 * k + imin];
                    sg ^= (uint8_t)(1 << imin);
                }
                block_signs[k] = sg & 127;
            }
            float mx = xval[0];
            for (int i = 1; i < 32; ++i) mx = std::max(mx, xval[i]);
            if (mx < 1e-15f) {
                scales[ib] = 0;
                continue;
            }
            float scale = make_qp_quants(32, kMaxQ + 1, xval, reinterpret_cast<uint8_t *>(L), weight);
            const float eff_max = scale * kMaxQ;
            if (eff_max <= 0) {
                scales[ib] = 0;
                continue;
            }
            float best = 0;
            for (int is = -6; is <= 6; ++is) {
                const float id = (2 * kMaxQ - 1 + is * 0.1f) / eff_max;
                const float this_scale = 1 / id;
                for (int k = 0; k < 4; ++k) {
                    for (int i = 0; i < 8; ++i) {
                        const int l = rne(0.5f * (id * xval[8 * k + i] - 1));
                        Laux[8 * k + i] = (int8_t)std::max(0, std::min(kMaxQ - 1, l));
                    }
                    int u = 0;
                    for (int i = 0; i < 8; ++i) u |= Laux[8 * k + i] << (2 * i);
                    if (S.map[u] < 0)
                        best_neighbour(S, S.nbr.data() - S.map[u] - 1, xval + 8 * k, waux + 8 * k, this_scale, Laux + 8 * k);
                }
                float sqx = 0, sq2 = 0;
                for (int i = 0; i < 32; ++i) {
                    const float q = 2 * Laux[i] + 1;
                    sqx += weight[i] * xval[i] * q;
                    sq2 += weight[i] * q * q;
                }
                if (sq2 > 0 && sqx * sqx > best * sq2) {
                    scale = sqx / sq2;
                    best = scale * sqx;
                    memcpy(L, Laux, 32);
                }
            }
            if (scale > 0) {
                const float id = 1 / scale;
                for (int k = 0; k < 4; ++k) {
                    int u = 0;
                    for (int i = 0; i < 8; ++i) {
                        const int l = std::max(0, std::min(kMaxQ - 1, rne(0.5f * (id * xval[8 * k + i] - 1))));
                        u |= l << (2 * i);
                    }
                    int row = S.map[u];
                    if (row < 0) row = best_neighbour(S, S.nbr.data() - S.map[u] - 1, xval + 8 * k, waux + 8 * k, scale, L + 8 * k);
                    for (int i = 0; i < 8; ++i) L[8 * k + i] = (int8_t)(((int)((S.grid[row] >> (8 * i)) & 0xff) - 1) / 2);
                }
                float sqx = 0, sq2 = 0;
                for (int i = 0; i < 32; ++i) {
                    const float q = 2 * L[i] + 1;
                    sqx += weight[i] * xval[i] * q;
                    sq2 += weight[i] * q * q;
                }
                if (sq2 > 0) scale = sqx / sq2;
            }
            if (scale < 0) {
                scale = -scale;
                for (int k = 0; k < 4; ++k) block_signs[k] = (uint8_t)((~block_signs[k]) & 127);
            }
            for (int k = 0; k < 4; ++k) {
                int u = 0;
                for (int i = 0; i < 8; ++i) u |= L[8 * k + i] << (2 * i);
                const int row = S.map[u];   // on the codebook by construction
                q2[2 * ib] |= (uint32_t)row << (8 * k);
                q2[2 * ib + 1] |= (uint32_t)block_signs[k] << (7 * k);
            }
            scales[ib] = scale;
            max_scale = std::max(max_scale, scale);
        }
        memset(y, 0, B_IQ2_XXS);
        if (!max_scale) continue;
        const float d = max_scale / 31;
        const uint16_t dh = to_f16(d);
        memcpy(y, &dh, 2);
        const float id = 1 / d;
        for (int ib = 0; ib < 8; ++ib) {
            const int l = std::max(0, std::min(15, rne(0.5f * (id * scales[ib] - 1))));
            q2[2 * ib + 1] |= (uint32_t)l << 28;
        }
        memcpy(y + 2, q2, 64);
    }
}

}  // namespace

extern "C" size_t moeb_quantize_weights(int32_t type, const float *src, void *dst, int64_t nrow, int64_t n_per_row,
                                        int32_t n_threads) {
    void (*row_fn)(const float *, uint8_t *, int64_t) = nullptr;
    int blk = 0;
    switch (type) {
        case MOEB_T_Q4_K:   row_fn = q4_k_row;   blk = 256; break;
        case MOEB_T_IQ2_S:  row_fn = iq2_s_row;  blk = 256; break;
        case MOEB_T_Q5_0:   row_fn = q5_0_row;   blk = 32;  break;
        case MOEB_T_IQ4_NL: row_fn = iq4_nl_row; blk = 32;  break;
        case MOEB_T_IQ2_XXS: row_fn = iq2_xxs_row; blk = 256; break;
        case MOEB_T_Q8_0:   row_fn = q8_0_row;   blk = 32;  break;
        default: return 0;
    }
    if (!src || !dst || nrow <= 0 || n_per_row <= 0 || n_per_row % blk) return 0;
    if (type == MOEB_T_IQ2_S) iq2s_search();
    if (type == MOEB_T_IQ2_XXS) iq2xxs_search();
    const int64_t rb = row_bytes(type, n_per_row);
    int nt = n_threads > 0 ? n_threads : (int)std::thread::hardware_concurrency();
    nt = (int)std::max<int64_t>(1, std::min<int64_t>(nt, nrow));
    auto work = [&](int t) {
        for (int64_t r = t; r < nrow; r += nt) row_fn(src + r * n_per_row, (uint8_t *)dst + r * rb, n_per_row);
    };
    if (nt == 1) {
        work(0);
    } else {
        std::vector<std::thread> th;
        for (int t = 0; t < nt; ++t) th.emplace_back(work, t);
        for (auto &t : th) t.join();
    }
    return (size_t)(nrow * rb);
}
