/*
 * TEST INFRASTRUCTURE — not product code.
 *
 * Shared plain-C description of one Gemma-4-style MoE FFN layer, used by the two CPU oracles:
 *   - oracle/ref_runner.cpp : the reference's own ggml-cpu graph (built from the reference sources
 *                              into oracle/_ref/), the "O1" oracle;
 *   - oracle/moe_oracle.c    : this repository's plain-C restatement of the same algorithm.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load either.
 *
 * Layer semantics follow build_moe_ffn (third_party/llama/src/llama-graph.cpp:1507-1851) with the
 * Gemma-4 arguments (third_party/llama/src/models/gemma4.cpp:409-425): softmax gating, top-k,
 * normalised weights (clamp 6.103515625e-5), merged gate_up MUL_MAT_ID, GeGLU (gate rows first),
 * down MUL_MAT_ID, per-expert down scale, weighting and the j-ordered add chain.
 * Precision classes follow the moe_dual residency mirror (ggml/include/ggml.h:1449-1471,
 * moert/cuda/ffn_moe.cu:101-104): a routed pair is "hot" iff
 *   0 <= exp_slot[e] < n_slots && slot_state[s] == 2 (READY) && slot_exp[s] == e,
 * and then uses the hot pool at slot s; otherwise it uses the cold pool at expert e.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (third_party/llama/ggml/include/ggml.h:390-432) */
enum {
    ORACLE_T_F32 = 0, ORACLE_T_F16 = 1, ORACLE_T_Q5_0 = 6, ORACLE_T_Q8_0 = 8, ORACLE_T_Q4_K = 12,
    ORACLE_T_Q8_K = 15, ORACLE_T_IQ2_XXS = 16, ORACLE_T_IQ4_NL = 20, ORACLE_T_IQ2_S = 22,
};

typedef struct oracle_layer {
    int32_t d_model, n_ff, n_expert, top_k, n_tokens;
    const float   *x;          /* [n_tokens][d_model]                                   */
    const float   *w_router;   /* [n_expert][d_model]                                   */
    const float   *b_router;   /* [n_expert] added to the logits, or NULL               */
    int32_t        n_slots;    /* hot pool capacity K (0 = no hot pool)                 */
    const int32_t *exp_slot;   /* [n_expert] expert -> slot or -1 (may be NULL if K==0) */
    const int32_t *slot_exp;   /* [K]                                                   */
    const int32_t *slot_state; /* [K]                                                   */
    int32_t        hot_type_gu, hot_type_down;
    const void    *hot_gu;     /* [K][2*n_ff rows][row bytes]                           */
    const void    *hot_down;   /* [K][d_model rows][row bytes]                          */
    const float   *s_hot;      /* [K] down scale or NULL                                */
    int32_t        cold_type_gu, cold_type_down;
    const void    *cold_gu;    /* [n_expert][2*n_ff rows][row bytes]                    */
    const void    *cold_down;  /* [n_expert][d_model rows][row bytes]                   */
    const float   *s_cold;     /* [n_expert] down scale or NULL                         */
    int32_t        n_threads;
    /* Conditional-parity inputs (port oracle only; the reference runner ignores them): when set,
     * the routed experts (ids_in, [n_tokens][top_k]) and/or the raw gate_up outputs of every
     * routed pair (gate_up_in, [n_tokens*top_k][2*n_ff], pair order) are taken as given instead
     * of being computed, so the later stages can be checked on exactly the inputs a tested
     * implementation fed them. */
    const int32_t *ids_in;
    const float   *gate_up_in;
    /* Router input when it differs from the experts' input x ([n_tokens][d_model], or NULL = x):
     * Gemma-4 routes on rms_norm(attn_out) / sqrt(d) * ffn_gate_inp_s and feeds the experts
     * rms_norm(attn_out) * ffn_pre_norm_2 (third_party/llama/src/models/gemma4.cpp:394-403). */
    const float   *x_router;
    /* 1: the GeGLU's GELU in tanh form evaluated in f32 (the CPU sidecar's, src/moe_sidecar.cpp:622-626)
     * instead of ggml-cpu's fp16 table; for attributing differences to that choice */
    int32_t        gelu_tanh;
} oracle_layer;

typedef struct oracle_layer_out {
    float   *logits;   /* [n_tokens][n_expert] or NULL                                       */
    float   *probs;    /* [n_tokens][n_expert] or NULL                                       */
    int32_t *ids;      /* [n_tokens][top_k]   or NULL  (the reference's top-k order)         */
    float   *weights;  /* [n_tokens][top_k]   or NULL  (normalised routing weights)          */
    float   *gate_up;  /* [n_tokens*top_k][2*n_ff] or NULL (raw gate_up per routed pair)      */
    float   *act;      /* [n_tokens*top_k][n_ff]   or NULL (GeGLU output per routed pair)     */
    float   *down;     /* [n_tokens*top_k][d_model] or NULL (scaled down output, pair order)  */
    float   *out;      /* [n_tokens][d_model]                                                */
} oracle_layer_out;

/* ---- the plain-C restatement (oracle/moe_oracle.c) ---- */
size_t  oracle_row_size(int32_t type, int64_t n);
void    oracle_dequantize_row(int32_t type, const void *src, float *dst, int64_t n);
/* activation quantisation to the weight type's vec_dot_type (Q8_K for Q4_K/IQ2_S, Q8_0 for
 * Q5_0/IQ4_NL), with the x86 reference semantics */
void    oracle_quantize_act(int32_t vec_dot_type, const float *x, void *y, int64_t n);
int32_t oracle_vec_dot_type(int32_t wtype);
float   oracle_vec_dot(int32_t wtype, int64_t n, const void *w_row, const void *x_q);
/* GeGLU with ggml-cpu's fp16-table GELU (ggml-cpu/vec.h:1414-1430) */
void    oracle_geglu(int64_t n, float *y, const float *gate, const float *up);
/* fp16 GELU table entry for the half bit pattern h (ggml-cpu.c:3792) */
uint16_t oracle_gelu_table(uint16_t h);
/* top-k in (value desc, index asc) order over one row */
void    oracle_topk(const float *v, int32_t n, int32_t k, int32_t *ids);
int     oracle_moe_layer(const oracle_layer *L, oracle_layer_out *o);
/* ggml_rms_norm over rows of n (ggml-cpu/ops.cpp, ggml_compute_forward_rms_norm_f32): the sum of
 * squares in double, scale = 1 / sqrtf(mean + eps) in float, y = x * scale; then y * s (ggml_scale)
 * and y * w[i] (ggml_mul with a [n] weight, w may be NULL), each an f32 product. The Gemma-4 block
 * norms: expert input s = 1, w = ffn_pre_norm_2; router input s = 1 / sqrtf(n), w = ffn_gate_inp_s;
 * output s = 1, w = ffn_post_norm_2 (third_party/llama/src/models/gemma4.cpp:394-427). */
void    oracle_rms_norm(const float *x, const float *w, float s, float *y, int64_t rows, int64_t n, float eps);
/* iq2s grid table used by the restatement (1024 packed 8-byte rows) */
const uint64_t *oracle_iq2s_grid(void);
const int8_t   *oracle_iq4nl_values(void);

/* ---- the reference harness (oracle/ref_runner.cpp over oracle/_ref/libggml_ref.so) ---- */
int     ref_init(void);
size_t  ref_row_size(int32_t type, int64_t n);
size_t  ref_quantize(int32_t type, const float *src, void *dst, int64_t nrow, int64_t n_per_row);
void    ref_dequantize_row(int32_t type, const void *src, float *dst, int64_t n);
void    ref_quantize_act(int32_t type, const float *x, void *y, int64_t n);
int32_t ref_vec_dot_type(int32_t wtype);
float   ref_vec_dot(int32_t wtype, int64_t n, const void *w_row, const void *x_q);
uint16_t ref_gelu_table(uint16_t h);
int     ref_moe_layer(const oracle_layer *L, oracle_layer_out *o);
int     ref_dense_ffn(const float *x, int64_t T, int64_t d, int64_t nff, int32_t gu_type, const void *w_gate,
                      const void *w_up, int32_t dn_type, const void *w_down, float *out, int n_threads);
size_t  ref_quantize_imatrix(int32_t type, const float *src, void *dst, int64_t nrow, int64_t n_per_row,
                             const float *imatrix);
void    ref_rms_norm(const float *x, const float *w, float s, float *y, int64_t rows, int64_t n, float eps);

#ifdef __cplusplus
}
#endif
#endif
