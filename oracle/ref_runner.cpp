// TEST INFRASTRUCTURE — not product code.
//
// Harness over the reference's own CPU implementation (ggml-base + ggml-cpu of the vendored
// llama.cpp fork, compiled from the reference sources into oracle/_ref/libggml_ref.so by
// oracle/Makefile). It exposes:
//   - the reference quantiser ggml_quantize_chunk (third_party/llama/ggml/src/ggml.c:7761),
//   - the reference dequantisers (type_traits.to_float, ggml/src/ggml-quants.c:442,1471,2471,2653),
//   - the CPU activation quantisers / vec_dots (ggml-cpu type_traits_cpu, arch/x86/quants.c),
//   - and ref_moe_layer: the "O1" oracle, a ggml-cpu graph that mirrors build_moe_ffn
//     (third_party/llama/src/llama-graph.cpp:1507-1851) with the Gemma-4 arguments
//     (third_party/llama/src/models/gemma4.cpp:409-425).
// Mixed precision uses the reference's partition semantics (moert/cuda/ffn_moe.cu:80-132): routed
// pairs are split into the hot and cold classes in ascending pair order, each class runs one
// MUL_MAT_ID over its compacted pair list, and the results are scattered back to pair order
// with the down scale applied once (ffn_moe.cu:158-176).

#include "moe_oracle.h"

#include "ggml.h"
#include "ggml-cpu.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

extern "C" uint16_t ggml_table_gelu_f16[1 << 16];   // ggml-cpu/vec.cpp:6, filled by ggml_cpu_init

namespace {

bool g_inited = false;

ggml_tensor * wrap(ggml_context * ctx, ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2, const void * data) {
    ggml_tensor * t = ggml_new_tensor_3d(ctx, type, ne0, ne1, ne2);
    t->data = const_cast<void *>(data);
    return t;
}

struct Ctx {
    ggml_context * meta = nullptr;   // no_alloc: tensors over caller memory
    ggml_context * work = nullptr;   // allocating: intermediates + graph work buffer
    Ctx(size_t work_bytes) {
        ggml_init_params pm = { ggml_tensor_overhead() * 64, nullptr, true };
        meta = ggml_init(pm);
        ggml_init_params pw = { work_bytes, nullptr, false };
        work = ggml_init(pw);
    }
    ~Ctx() { ggml_free(meta); ggml_free(work); }
};

bool is_hot(const oracle_layer * L, int e, int * slot) {
    if (L->n_slots <= 0 || !L->exp_slot) return false;
    const int s = L->exp_slot[e];
    if (s >= 0 && s < L->n_slots && L->slot_state[s] == 2 && L->slot_exp[s] == e) { *slot = s; return true; }
    return false;
}

}  // namespace

extern "C" int ref_init(void) {
    if (!g_inited) {
        ggml_cpu_init();
        g_inited = true;
    }
    return 1;
}

extern "C" size_t ref_row_size(int32_t type, int64_t n) { return ggml_row_size((ggml_type) type, n); }

extern "C" size_t ref_quantize(int32_t type, const float * src, void * dst, int64_t nrow, int64_t n_per_row) {
    ref_init();
    return ggml_quantize_chunk((ggml_type) type, src, dst, 0, nrow, n_per_row, nullptr);
}

// the same with an importance matrix (f32 [n_per_row]); the types ggml quantises only with one
// (IQ2_XXS, IQ2_XS, IQ1_S: ggml.c:7753-7772) need it
extern "C" size_t ref_quantize_imatrix(int32_t type, const float * src, void * dst, int64_t nrow, int64_t n_per_row,
                                       const float * imatrix) {
    ref_init();
    return ggml_quantize_chunk((ggml_type) type, src, dst, 0, nrow, n_per_row, imatrix);
}

extern "C" void ref_dequantize_row(int32_t type, const void * src, float * dst, int64_t n) {
    ref_init();
    ggml_get_type_traits((ggml_type) type)->to_float(src, dst, n);
}

extern "C" void ref_quantize_act(int32_t type, const float * x, void * y, int64_t n) {
    ref_init();
    ggml_get_type_traits_cpu((ggml_type) type)->from_float(x, y, n);
}

extern "C" int32_t ref_vec_dot_type(int32_t wtype) {
    ref_init();
    return (int32_t) ggml_get_type_traits_cpu((ggml_type) wtype)->vec_dot_type;
}

extern "C" float ref_vec_dot(int32_t wtype, int64_t n, const void * w_row, const void * x_q) {
    ref_init();
    float s = 0.0f;
    ggml_get_type_traits_cpu((ggml_type) wtype)->vec_dot((int) n, &s, 0, w_row, 0, x_q, 0, 1);
    return s;
}

extern "C" uint16_t ref_gelu_table(uint16_t h) {
    ref_init();
    return ggml_table_gelu_f16[h];
}

// One class of routed pairs through gate_up -> GeGLU -> down, as MUL_MAT_ID over the compacted
// pair list (one "token" per pair, n_used = 1).
static void run_class(const oracle_layer * L, int type_gu, int type_down, const void * w_gu, const void * w_down,
                      int n_w, const std::vector<int> & pairs, const std::vector<int> & wid,
                      const float * scale, std::vector<float> & gate_up_pp, std::vector<float> & act_pp,
                      std::vector<float> & down_pp) {
    const int n = (int) pairs.size();
    if (n == 0) return;
    const int d = L->d_model, nff = L->n_ff, k = L->top_k;
    const size_t work = (size_t) n * (2 * nff + nff + 2 * d + 64) * sizeof(float) * 2
                      + (size_t) n * (d + nff) * 2 + (64u << 20);
    Ctx c(work);
    ggml_tensor * wgu = wrap(c.meta, (ggml_type) type_gu, d, 2 * nff, n_w, w_gu);
    ggml_tensor * wdn = wrap(c.meta, (ggml_type) type_down, nff, d, n_w, w_down);
    ggml_tensor * cur = ggml_new_tensor_3d(c.work, GGML_TYPE_F32, d, 1, n);
    ggml_tensor * ids = ggml_new_tensor_2d(c.work, GGML_TYPE_I32, 1, n);
    for (int i = 0; i < n; ++i) {
        const int t = pairs[i] / k;
        memcpy((float *) cur->data + (size_t) i * d, L->x + (size_t) t * d, sizeof(float) * d);
        ((int32_t *) ids->data)[i] = wid[i];
    }
    ggml_tensor * gu = ggml_mul_mat_id(c.work, wgu, cur, ids);                    // [2nff, 1, n]
    ggml_tensor * g  = ggml_view_3d(c.work, gu, nff, 1, n, gu->nb[1], gu->nb[2], 0);
    ggml_tensor * u  = ggml_view_3d(c.work, gu, nff, 1, n, gu->nb[1], gu->nb[2], nff * gu->nb[0]);
    ggml_tensor * a  = ggml_geglu_split(c.work, g, u);                             // [nff, 1, n]
    ggml_tensor * y  = ggml_mul_mat_id(c.work, wdn, a, ids);                       // [d, 1, n]
    if (scale) {
        ggml_tensor * s = ggml_new_tensor_3d(c.work, GGML_TYPE_F32, 1, 1, n);
        for (int i = 0; i < n; ++i) ((float *) s->data)[i] = scale[wid[i]];
        y = ggml_mul(c.work, y, s);                                               // apply_scale, moe_dual.cpp:91
    }
    ggml_cgraph * gf = ggml_new_graph(c.work);
    ggml_build_forward_expand(gf, y);
    ggml_graph_compute_with_ctx(c.work, gf, L->n_threads > 0 ? L->n_threads : 1);
    for (int i = 0; i < n; ++i) {
        const int p = pairs[i];
        memcpy(&gate_up_pp[(size_t) p * 2 * nff], (const char *) gu->data + (size_t) i * gu->nb[2], sizeof(float) * 2 * nff);
        memcpy(&act_pp[(size_t) p * nff], (const char *) a->data + (size_t) i * a->nb[2], sizeof(float) * nff);
        memcpy(&down_pp[(size_t) p * d], (const char *) y->data + (size_t) i * y->nb[2], sizeof(float) * d);
    }
}

extern "C" int ref_moe_layer(const oracle_layer * L, oracle_layer_out * o) {
    ref_init();
    const int d = L->d_model, E = L->n_expert, k = L->top_k, T = L->n_tokens, nff = L->n_ff;
    const int nth = L->n_threads > 0 ? L->n_threads : 1;

    // ---- stage A: router -> softmax -> top-k -> weights (llama-graph.cpp:1530-1650) ----
    std::vector<int32_t> ids((size_t) T * k);
    std::vector<float>   wts((size_t) T * k);
    {
        Ctx c((size_t) T * E * 4 * 8 + (size_t) T * d * 4 + (16u << 20));
        ggml_tensor * x  = wrap(c.meta, GGML_TYPE_F32, d, T, 1, L->x_router ? L->x_router : L->x);
        ggml_tensor * wr = wrap(c.meta, GGML_TYPE_F32, d, E, 1, L->w_router);
        x  = ggml_reshape_2d(c.meta, x, d, T);
        wr = ggml_reshape_2d(c.meta, wr, d, E);
        ggml_tensor * logits = ggml_mul_mat(c.work, wr, x);                                   // [E, T]
        if (L->b_router) {
            ggml_tensor * b = wrap(c.meta, GGML_TYPE_F32, E, 1, 1, L->b_router);
            logits = ggml_add(c.work, logits, ggml_reshape_1d(c.meta, b, E));
        }
        ggml_tensor * probs = ggml_soft_max(c.work, logits);                                  // [E, T]
        ggml_tensor * sel   = ggml_argsort_top_k(c.work, probs, k);                           // [k, T]
        ggml_tensor * w     = ggml_get_rows(c.work, ggml_reshape_3d(c.work, probs, 1, E, T), sel);
        w = ggml_reshape_2d(c.work, w, k, T);
        ggml_tensor * wsum = ggml_sum_rows(c.work, w);
        wsum = ggml_clamp(c.work, wsum, 6.103515625e-5f, INFINITY);
        w = ggml_div(c.work, w, wsum);
        ggml_cgraph * gf = ggml_new_graph(c.work);
        ggml_build_forward_expand(gf, logits);
        ggml_build_forward_expand(gf, probs);
        ggml_build_forward_expand(gf, sel);
        ggml_build_forward_expand(gf, w);
        ggml_graph_compute_with_ctx(c.work, gf, nth);
        for (int t = 0; t < T; ++t) {
            for (int j = 0; j < k; ++j) {
                ids[(size_t) t * k + j] = *(const int32_t *) ((const char *) sel->data + t * sel->nb[1] + j * sel->nb[0]);
                wts[(size_t) t * k + j] = *(const float *) ((const char *) w->data + t * w->nb[1] + j * w->nb[0]);
            }
            if (o->logits) memcpy(o->logits + (size_t) t * E, (const char *) logits->data + t * logits->nb[1], sizeof(float) * E);
            if (o->probs)  memcpy(o->probs  + (size_t) t * E, (const char *) probs->data  + t * probs->nb[1],  sizeof(float) * E);
        }
    }
    if (o->ids)     memcpy(o->ids, ids.data(), sizeof(int32_t) * ids.size());
    if (o->weights) memcpy(o->weights, wts.data(), sizeof(float) * wts.size());

    // ---- stage B: partition by residency, then one MUL_MAT_ID chain per class ----
    const int P = T * k;
    std::vector<int> hot_p, hot_w, cold_p, cold_w;
    for (int p = 0; p < P; ++p) {
        const int e = ids[p];
        int s = -1;
        if (is_hot(L, e, &s)) { hot_p.push_back(p); hot_w.push_back(s); }
        else                  { cold_p.push_back(p); cold_w.push_back(e); }
    }
    std::vector<float> gate_up_pp((size_t) P * 2 * nff), act_pp((size_t) P * nff), down_pp((size_t) P * d);
    run_class(L, L->hot_type_gu, L->hot_type_down, L->hot_gu, L->hot_down, L->n_slots, hot_p, hot_w, L->s_hot,
              gate_up_pp, act_pp, down_pp);
    run_class(L, L->cold_type_gu, L->cold_type_down, L->cold_gu, L->cold_down, E, cold_p, cold_w, L->s_cold,
              gate_up_pp, act_pp, down_pp);
    if (o->gate_up) memcpy(o->gate_up, gate_up_pp.data(), sizeof(float) * gate_up_pp.size());
    if (o->act)     memcpy(o->act, act_pp.data(), sizeof(float) * act_pp.size());
    if (o->down)    memcpy(o->down, down_pp.data(), sizeof(float) * down_pp.size());

    // ---- stage C: weighting and the j-ordered add chain (llama-graph.cpp:1812-1848) ----
    {
        Ctx c((size_t) P * d * 4 * 3 + (16u << 20));
        ggml_tensor * ex = wrap(c.meta, GGML_TYPE_F32, d, k, T, down_pp.data());
        ggml_tensor * w  = wrap(c.meta, GGML_TYPE_F32, 1, k, T, wts.data());
        ggml_tensor * y  = ggml_mul(c.work, ex, w);
        ggml_tensor * acc = ggml_view_2d(c.work, y, d, T, y->nb[2], 0);
        for (int j = 1; j < k; ++j)
            acc = ggml_add(c.work, acc, ggml_view_2d(c.work, y, d, T, y->nb[2], j * y->nb[1]));
        if (k == 1) acc = ggml_cont(c.work, acc);
        ggml_cgraph * gf = ggml_new_graph(c.work);
        ggml_build_forward_expand(gf, acc);
        ggml_graph_compute_with_ctx(c.work, gf, nth);
        for (int t = 0; t < T; ++t)
            memcpy(o->out + (size_t) t * d, (const char *) acc->data + t * acc->nb[1], sizeof(float) * d);
    }
    return 1;
}

// The Gemma-4 dense MLP's FFN nodes as build_ffn adds them with GELU / PAR and no biases or scales
// (llama-graph.cpp:1316-1390, gemma4.cpp:382-387): gate = W_gate x, up = W_up x, a = geglu_split(gate,
// up), out = W_down a. Weights in ggml layout ([rows][row bytes]); x and out f32 [T][d].
extern "C" int ref_dense_ffn(const float * x, int64_t T, int64_t d, int64_t nff, int32_t gu_type, const void * w_gate,
                             const void * w_up, int32_t dn_type, const void * w_down, float * out, int n_threads) {
    ref_init();
    Ctx c((size_t) T * (3 * nff + 2 * d) * 4 * 4 + (64u << 20));
    ggml_tensor * xt = ggml_reshape_2d(c.meta, wrap(c.meta, GGML_TYPE_F32, d, T, 1, x), d, T);
    ggml_tensor * wg = ggml_reshape_2d(c.meta, wrap(c.meta, (ggml_type) gu_type, d, nff, 1, w_gate), d, nff);
    ggml_tensor * wu = ggml_reshape_2d(c.meta, wrap(c.meta, (ggml_type) gu_type, d, nff, 1, w_up), d, nff);
    ggml_tensor * wd = ggml_reshape_2d(c.meta, wrap(c.meta, (ggml_type) dn_type, nff, d, 1, w_down), nff, d);
    ggml_tensor * up = ggml_mul_mat(c.work, wu, xt);
    ggml_tensor * gate = ggml_mul_mat(c.work, wg, xt);
    ggml_tensor * a = ggml_geglu_split(c.work, gate, up);
    ggml_tensor * y = ggml_mul_mat(c.work, wd, a);
    ggml_cgraph * gf = ggml_new_graph(c.work);
    ggml_build_forward_expand(gf, y);
    ggml_graph_compute_with_ctx(c.work, gf, n_threads);
    for (int64_t t = 0; t < T; ++t) memcpy(out + t * d, (const char *) y->data + t * y->nb[1], sizeof(float) * d);
    return 1;
}

// ggml_rms_norm over `rows` rows of n values, then ggml_scale by s (when s != 1) and ggml_mul by the
// [n] weight w (when given): the reference's own nodes, as the Gemma-4 block builds them
extern "C" void ref_rms_norm(const float * x, const float * w, float s, float * y, int64_t rows, int64_t n, float eps) {
    ref_init();
    Ctx c((size_t) rows * n * 4 * 4 + (4u << 20));
    ggml_tensor * xt = wrap(c.meta, GGML_TYPE_F32, n, rows, 1, x);
    xt = ggml_reshape_2d(c.meta, xt, n, rows);
    ggml_tensor * yt = ggml_rms_norm(c.work, xt, eps);
    if (s != 1.0f) yt = ggml_scale(c.work, yt, s);
    if (w) yt = ggml_mul(c.work, yt, wrap(c.meta, GGML_TYPE_F32, n, 1, 1, w));
    ggml_cgraph * gf = ggml_new_graph(c.work);
    ggml_build_forward_expand(gf, yt);
    ggml_graph_compute_with_ctx(c.work, gf, 1);
    for (int64_t r = 0; r < rows; ++r)
        memcpy(y + r * n, (const char *) yt->data + r * yt->nb[1], sizeof(float) * n);
}
