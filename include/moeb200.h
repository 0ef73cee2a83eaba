/*
 * moeb200.h — B200-native entry points of the MoE-FFN hot path (libmoeb200.so).
 *
 * The Gemma-4 MoE FFN layer as LLapis computes it through GGML_OP_MOE_DUAL / GGML_OP_MUL_MAT_ID
 * (third_party/llama/src/llama-graph.cpp:1507-1851, gemma4.cpp:409-425):
 *   router logits (f32) [+ bias] -> softmax -> top-k (value desc, lowest index on ties)
 *   -> normalised weights -> per-expert dispatch (histogram, exclusive scan, stable permutation)
 *   -> grouped gate_up with on-the-fly Q4_K / IQ2_S dequantisation (activations as Q8_K)
 *   -> GeGLU (ggml-cpu fp16-table GELU) -> down projection (Q5_0 / IQ4_NL, activations as Q8_0)
 *   -> per-expert down scale -> routing-weighted, slot-ordered combine.
 * Two precision classes live in HBM, selected per routed pair by the moe_dual residency mirror:
 * a pair is hot iff 0 <= exp_slot[e] < n_slots, slot_state[slot] == 2 and slot_exp[slot] == e
 * (moert/cuda/ffn_moe.cu:101-104); hot pairs read the hot pool at `slot`, cold pairs the cold
 * pool at `e`.
 *
 * Conventions: device pointers unless stated; ggml layouts (a weight pool is
 * [slots][rows][row bytes], activations are [tokens][features] f32 rows); `stream` is a
 * cudaStream_t passed as void*. Every entry returns 0 on success or a negative MOEB_E* code;
 * moeb_last_error() gives the message. Nothing falls back to the CPU: without a usable sm_100
 * device every compute entry fails with MOEB_ENODEV.
 */
#ifndef MOEB200_H
#define MOEB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    MOEB_OK = 0,
    MOEB_EINVAL = -1,    /* bad argument or shape                                    */
    MOEB_ENODEV = -2,    /* no sm_100 device / CUDA unavailable                      */
    MOEB_ECUDA = -3,     /* a CUDA runtime call failed                               */
    MOEB_ESPACE = -4,    /* workspace too small                                      */
    MOEB_EDEVICE = -5,   /* a kernel reported an error (bounded wait gave up, bad id) */
    MOEB_ETYPE = -6,     /* weight type not supported on this path                   */
};

/* ggml type ids accepted as weight types (third_party/llama/ggml/include/ggml.h:390-432) */
enum { MOEB_T_Q5_0 = 6, MOEB_T_Q4_K = 12, MOEB_T_IQ4_NL = 20, MOEB_T_IQ2_S = 22 };
/* further expert types the product files use; so far moeb_dequantize and moeb_row_size only */
enum { MOEB_T_Q8_0 = 8, MOEB_T_IQ2_XXS = 16 };

/* One HBM-resident precision class: merged gate_up [n][2*n_ff rows][row(d_model)] and
 * down [n][d_model rows][row(n_ff)], each in ggml block layout. */
typedef struct moeb_pool {
    int32_t     type_gu;     /* MOEB_T_Q4_K or MOEB_T_IQ2_S                  */
    int32_t     type_down;   /* MOEB_T_Q5_0 or MOEB_T_IQ4_NL                 */
    int32_t     n;           /* experts (cold pool) or slots (hot pool)      */
    int32_t     _pad;
    const void *w_gu;
    const void *w_down;
    const float *s_down;     /* f32 [n] down scale (ffn_down_exps_s) or NULL */
} moeb_pool;

/* One MoE layer (replaces the per-layer tensors build_moe_ffn reads). */
typedef struct moeb_layer {
    int32_t        d_model, n_ff, n_expert, top_k;
    const float   *w_router;   /* f32 [n_expert][d_model] (ffn_gate_inp)                */
    const float   *b_router;   /* f32 [n_expert] added to the logits, or NULL           */
    moeb_pool      hot;        /* n = slot count K (may be 0)                           */
    moeb_pool      cold;       /* n = n_expert (may be 0 when every expert is hot)      */
    const int32_t *exp_slot;   /* i32 [n_expert] (NULL when hot.n == 0)                 */
    const int32_t *slot_exp;   /* i32 [K]                                               */
    const int32_t *slot_state; /* i32 [K], 2 = READY                                    */
} moeb_layer;

/* Optional per-call outputs for inspection / parity (any pointer may be NULL). */
typedef struct moeb_layer_aux {
    float   *logits;     /* f32 [T][n_expert] router logits (+ bias)                          */
    int32_t *ids;        /* i32 [T][top_k] selected experts, (value desc, index asc)          */
    float   *weights;    /* f32 [T][top_k] normalised routing weights                         */
    int32_t *counts;     /* i32 [n_expert] routed pairs per expert (histogram)                */
    int32_t *offsets;    /* i32 [n_expert + 1] exclusive scan of counts                       */
    int32_t *perm;       /* i32 [T*top_k] pair indices p = t*top_k + j grouped by expert, stable */
    float   *gate_up;    /* f32 [T*top_k][2*n_ff] raw gate_up per routed pair                 */
    float   *down;       /* f32 [T*top_k][d_model] scaled down output per routed pair         */
} moeb_layer_aux;

/* Library and device setup. moeb_init loads the format tables into the current device (once per
 * device; also done lazily by the first compute call on a device). */
int         moeb_init(void);
const char *moeb_last_error(void);
const char *moeb_version(void);
/* Reads and clears the device error word (bit 1: a bounded wait gave up; 2: expert id out of
 * range; 4: a capacity limit was exceeded; 16: a GeGLU output beyond the fp16 operand range of
 * the prefill down GEMM, |value| > 65504). */
int32_t     moeb_device_error(void *stream);

/* Workspace bytes moeb_layer_forward needs for n_tokens tokens (the decode path needs one 8-token
 * chunk's worth for any n_tokens; the prefill path grows with n_tokens, dominated by the f32 down
 * outputs of every routed pair: n_tokens * top_k * d_model * 4 bytes). */
size_t moeb_layer_workspace_size(const moeb_layer *L, int32_t n_tokens);

/* The path moeb_layer_forward takes for n_tokens tokens of this layer (new, an inspection entry):
 * 0 the fused decode kernel (8-token chunks), 1 the prefill kernels; a negative MOEB_E* code for a
 * layer moeb_layer_forward would refuse. Layers whose decode kernel does not fit in an SM's shared
 * memory (n_ff above ~1.5K at d_model 2816, e.g. the Gemma-4 dense MLP's 2112) take the prefill
 * path at every batch size. */
int32_t moeb_layer_path(const moeb_layer *L, int32_t n_tokens);

/* One whole MoE layer, router to combine (new; the graph-level unit the benchmark measures).
 * x: f32 [n_tokens][d_model]; out: f32 [n_tokens][d_model]. The workspace must stay untouched
 * until the stream reaches the end of the call. Kernels are chained with programmatic dependent
 * launch; the call is stream-ordered and capturable in a CUDA graph.
 * Batches below the prefill threshold run the decode path (one fused cooperative kernel per
 * 8 tokens, integer dot-product GEMVs); larger ones the prefill path (grouped GEMMs on the
 * tcgen05 tensor cores). Both reproduce the reference's integer block dot products. */
int moeb_layer_forward(const moeb_layer *L, const float *x, int32_t n_tokens, float *out,
                       const moeb_layer_aux *aux, void *workspace, size_t workspace_bytes, void *stream);

/* The norms around the Gemma-4 MoE block (third_party/llama/src/models/gemma4.cpp:394-427), device
 * pointers to f32 [d_model] vectors, 16-byte aligned:
 *   expert input = rms_norm(x) * pre_norm                      (ffn_pre_norm_2, gemma4.cpp:394-396)
 *   router input = rms_norm(x) * (1 / sqrtf(d_model)) * router_scale   (ffn_gate_inp_s, :399-402)
 *   out          = rms_norm(moe(expert input)) * post_norm    (ffn_post_norm_2, :423-425)
 * rms_norm(v) = v * (1 / sqrt(mean(v^2) + eps)) with ggml_rms_norm's arithmetic. */
typedef struct moeb_norms {
    const float *pre_norm;
    const float *router_scale;
    const float *post_norm;
    float        eps;          /* f_norm_rms_eps, >= 0 */
    int32_t      _pad;
} moeb_norms;

/* moeb_layer_forward with the Gemma-4 block norms fused in (new; the reference runs them as separate
 * graph nodes around build_moe_ffn): x is the block input (attn_out), out the normed MoE output
 * that the host adds to the dense MLP branch. Same paths, workspace size and aux outputs as
 * moeb_layer_forward (aux->logits are the logits of the router input, aux->gate_up and
 * aux->down are computed from the expert input; out is after the output norm). The norms add no
 * launch: the decode kernel takes the row scales from the squares of its own loads of x (the
 * router's row scale factored out of its dot product: the logits equal the reference's to f32
 * rounding, as their summation order already makes them) and norms each token's output row after
 * its last block is combined; the prefill path's first kernel computes the row scales and the
 * expert input's Q8_K rows, the router forms its input value by value as it stages x, and the
 * combine kernel applies the output norm. d_model <= 4096. */
int moeb_layer_forward_gemma4(const moeb_layer *L, const moeb_norms *norms, const float *x, int32_t n_tokens,
                              float *out, const moeb_layer_aux *aux, void *workspace, size_t workspace_bytes,
                              void *stream);

/* The feed-forward part of a Gemma-4 MoE block (new; third_party/llama/src/models/gemma4.cpp:376-431):
 *   mlp = rms_norm(x) * ffn_norm -> build_ffn (GELU, PAR) -> rms_norm * ffn_post_norm_1   (dense branch)
 *   moe = moeb_layer_forward_gemma4(moe, moe_norms, x)                                     (MoE branch)
 *   out = moe + mlp                                                                        (ggml_add)
 * The dense MLP is passed as a one-expert layer (top_k 1, one hot slot holding [gate rows; up rows]
 * and down, zero router weights with a bias putting every token on expert 0: its softmax weight is
 * then exactly 1.0) with mlp_norms = {ffn_norm, any non-null router_scale (unused: the router weights
 * are zero), ffn_post_norm_1}. With a side_stream the dense branch runs there, concurrently with the
 * MoE branch on stream (fork / join through events, capturable in a CUDA graph); with side_stream
 * NULL both run on stream in turn. Calls on one device issued from several host threads at once are
 * serialised on the host while they enqueue. The workspace (moeb_ffn_block_workspace_size) holds
 * both branches' workspaces and the dense branch's output. */
/* Row-wise rms_norm followed by the reference's optional scale and mul nodes (new; ggml_rms_norm
 * then ggml_scale and ggml_mul, as the Gemma-4 block applies them, gemma4.cpp:394-402, :423-425):
 * out = ((x * s) * scale) * w per row, s = 1 / sqrt(mean(x^2) + eps), each product rounded to f32;
 * scale 1 skips the scale node, w NULL the mul node. x, out: f32 [rows][d], 16-byte aligned, d a
 * multiple of 4; out may equal x. The expert-parallel layer norms its tokens with it before the
 * dispatch and after the cross-rank combine. */
int moeb_rms_norm(const float *x, int32_t rows, int32_t d, const float *w, float scale, float eps, float *out,
                  void *stream);

size_t moeb_ffn_block_workspace_size(const moeb_layer *moe, const moeb_layer *mlp, int32_t n_tokens);
int moeb_ffn_block_gemma4(const moeb_layer *moe, const moeb_norms *moe_norms, const moeb_layer *mlp,
                          const moeb_norms *mlp_norms, const float *x, int32_t n_tokens, float *out,
                          void *workspace, size_t workspace_bytes, void *stream, void *side_stream);

/* The two halves of the layer, for expert-parallel hosts (new; the reference runs the router and
 * the expert matmuls as separate graph nodes, llama-graph.cpp:1530-1613 and :1689-1848).
 *  moeb_layer_route: router logits (f32 [n_tokens][n_expert], caller memory), top-k ids
 *    (i32 [n_tokens][top_k]) and normalised weights (f32 [n_tokens][top_k]). With a workspace of
 *    moeb_route_workspace_size bytes the logits GEMM splits K four ways (more CTAs for the same
 *    tokens, partial sums added in order); with workspace NULL it runs in one part.
 *  moeb_layer_forward_routed: the expert half for rows whose routing is given: out[r] =
 *    sum_j weights[r][j] * down(GeGLU(gate_up(x[r]))) over the slots j with ids[r][j] >= 0, in
 *    slot order; negative ids mark experts that live elsewhere. Runs the prefill kernels for any
 *    n_rows >= 1 (the layer needs the prefill shapes); workspace from moeb_routed_workspace_size. */
int    moeb_layer_route(const moeb_layer *L, const float *x, int32_t n_tokens, float *logits, int32_t *ids,
                        float *weights, void *workspace, size_t workspace_bytes, void *stream);
size_t moeb_route_workspace_size(const moeb_layer *L, int32_t n_tokens);
size_t moeb_routed_workspace_size(const moeb_layer *L, int32_t n_rows);
int    moeb_layer_forward_routed(const moeb_layer *L, const float *x, int32_t n_rows, const int32_t *ids,
                                 const float *weights, float *out, void *workspace, size_t workspace_bytes,
                                 void *stream);
/* The same expert half on rows already quantised to Q8_K (new): xq is [n_rows][d_model / 256] ggml
 * block_q8_K (d f32 | qs[256] | bsums[16] i16, 292 bytes a block), as moeb_quantize_act(MOEB_T_Q8_K)
 * writes it, 16-byte aligned. The experts consume exactly these bytes, so an expert-parallel host can
 * send them in place of f32 rows (3,212 bytes a 2816-wide row instead of 11,264) with identical
 * results. */
int    moeb_layer_forward_routed_q8k(const moeb_layer *L, const void *xq, int32_t n_rows, const int32_t *ids,
                                     const float *weights, float *out, void *workspace, size_t workspace_bytes,
                                     void *stream);

/* Sets the smallest batch that moeb_layer_forward runs on the prefill path (default 64; values
 * <= 0 leave it unchanged) and returns the previous value. Process-wide. No counterpart in the
 * reference (its ggml-cuda backend picks mul_mat_vec_q or mul_mat_q by batch size internally,
 * ggml-cuda.cu). Layers whose shape the prefill kernels do not cover (n_ff not a multiple of 64,
 * d_model not a multiple of 128, d_model > 4096 or n_ff > 4096) always take the decode path; layers
 * whose decode kernel does not fit in shared memory always take the prefill path. */
int32_t moeb_set_prefill_min_tokens(int32_t n_tokens);

/* Sets the bound on the mean routed pairs per expert (top_k x n_tokens / n_expert) below which a
 * batch on the prefill path runs gate_up on the mid-size kernels instead of the tcgen05 GEMM (default 48;
 * values <= 0 leave it unchanged; 1 turns the mid-size kernels off) and returns the previous value.
 * Process-wide. The mid-size kernels stream each routed expert's rows once and multiply the
 * weights' own integer codes (warp-level int8 MMAs) by every 8-pair block of its tokens, so their
 * cost follows the weight bytes, where the tcgen05 path converts every weight element into an
 * fp16 operand. Layers whose shape they do not cover fall back to the tcgen05 path. */
int32_t moeb_set_mid_max_pairs(int32_t pairs_per_expert);

/* The same bound for the down projection (default 16): the two projections choose their kernels
 * independently (both hand over the gate_up rows in the same slot-order buffer). */
int32_t moeb_set_mid_max_pairs_down(int32_t pairs_per_expert);

/* Profiling of the prefill path (no counterpart in the reference): while enabled, every prefill
 * forward on the current device records CUDA events around its nine kernels (router, top-k,
 * dispatch, activation quantisation, operand gather, gate_up, GeGLU, down, combine) on the
 * caller's stream. Events
 * between kernels keep them from overlapping, so use it on a separate measurement pass.
 * moeb_prefill_profile_read waits for the last profiled call and writes up to n durations (ms). */
int moeb_prefill_profile(int32_t enable);
int moeb_prefill_profile_read(float *ms, int32_t n);

/* Allocation-free variant of moeb_layer_forward. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory where they call the layer: hosts whose own
 * memory manager has reserved all of HBM up front and forbids stray allocations (an inference
 * server carving the device into its own pools), plug-ins loaded into such a process that must not
 * disturb its allocator, and latency-critical paths that cannot afford cudaMalloc's implicit
 * device synchronisation. The caller passes only inputs and outputs; the workspace lives in a
 * library-owned static device array of MOEB_STATIC_SCRATCH_BYTES, held by every GPU that loads
 * the library until the process exits. It allocates no device memory and calls no allocating
 * library routine.
 *
 * Limits and rules:
 *  - it always runs the decode path (chunks of 8 tokens), whose workspace is one chunk's worth
 *    for any n_tokens; a layer whose chunk workspace exceeds MOEB_STATIC_SCRATCH_BYTES is
 *    rejected with MOEB_ESPACE (the Gemma-4 26B-A4B layer needs about 2.2 MB);
 *  - the first call on a device does one-time set-up there (format tables, the device address of
 *    the static array); make that first call before any stream capture on that device;
 *  - the device address is kept for the life of the process: do not use this entry on a device
 *    after cudaDeviceReset (or any other re-creation of its primary context), which reloads the
 *    library's module there and leaves the kept address pointing at freed memory;
 *  - all calls share the one array per device and it keeps the last call's contents: calls that
 *    overlap on the GPU (different streams, or different host threads, on the same device) race.
 *    Nothing in it needs clearing between calls; every byte a forward reads it writes first. */
#define MOEB_STATIC_SCRATCH_BYTES (4u << 20)
int moeb_layer_forward_static(const moeb_layer *L, const float *x, int32_t n_tokens, float *out, void *stream);

/* Binds the weight pools that moert_ffn_moe(il, kind) reads (the reference trampoline lends its
 * w_hot / w_cold tensors through the mm vtable instead, moe-dual.cu:74-94). hot/cold: device
 * pools in ggml layout [n][d_out][row(d_in)] of type hot_type / cold_type. */
int moeb_bind_pools(int32_t il, int32_t kind, const void *w_hot, int32_t hot_type, int32_t n_hot,
                    const void *w_cold, int32_t cold_type, int32_t n_cold);

/* Router epilogue alone: softmax / top-k / weights over given logits f32 [T][n_expert]
 * (the index-parity check feeds the reference's logits through this). */
int moeb_router_topk(const float *logits, int32_t n_tokens, int32_t n_expert, int32_t top_k,
                     int32_t *ids, float *weights, void *stream);

/* Dispatch alone: ids i32 [T][top_k] -> counts [n_expert], offsets [n_expert+1], perm [T*top_k]
 * (histogram, exclusive scan, stable permutation; mmid.cu:28 / ggml-cpu.c:1613-1626). */
int moeb_dispatch(const int32_t *ids, int32_t n_tokens, int32_t top_k, int32_t n_expert,
                  int32_t *counts, int32_t *offsets, int32_t *perm, void *stream);

/* Weight dequantisation to f32 rows (bit-exact with ggml's dequantize_row_*): Q4_K, IQ2_S, Q5_0,
 * IQ4_NL, IQ2_XXS, Q8_0. */
int moeb_dequantize(int32_t type, const void *src, float *dst, int64_t n_rows, int64_t n_per_row, void *stream);

/* Activation quantisation of f32 rows to the vec_dot type of `wtype` (Q8_K for Q4_K/IQ2_S, Q8_0
 * for Q5_0/IQ4_NL), bit-exact with ggml-cpu on x86. */
int moeb_quantize_act(int32_t wtype, const float *x, void *dst, int64_t n_rows, int64_t n_per_row, void *stream);

/* ---- host-side weight quantiser (CPU, multi-threaded) ----
 * Restates ggml_quantize_chunk without an importance matrix (third_party/llama/ggml/src/ggml.c:7761)
 * for the four expert types and Q8_0, and for IQ2_XXS with a uniform one (ggml requires one there);
 * output bytes are identical to the reference quantiser's. src: host
 * f32 [nrow][n_per_row]; dst: host. n_threads <= 0 uses every online CPU. Returns bytes written,
 * or 0 on a bad type/shape. */
size_t moeb_quantize_weights(int32_t type, const float *src, void *dst, int64_t nrow, int64_t n_per_row,
                             int32_t n_threads);
size_t moeb_row_size(int32_t type, int64_t n_per_row);

/* ---- Expert loading from files into the class pools (new; the reference's host loads the same
 * tensors through ggml's GGUF reader, third_party/llama/ggml/src/gguf.cpp, and the hot class's
 * pages through its expert store and memory manager, moert/include/moert/store.h and memmgr.h).
 * A Gemma-4 layer's stacked expert tensors in a GGUF (blk.<il>.ffn_gate_up_exps.weight
 * [n_embd, 2*n_ff, E], blk.<il>.ffn_down_exps.weight [n_ff, n_embd, E]) are laid out exactly as a
 * cold pool ([E][rows][row bytes]); the hot pool's slots are filled page by page from a store
 * (include/moert_store.h). Host functions; the copies run on `stream` and have completed when a
 * loader returns. */

/* GGUF tensor directory: header, key/values (arrays skipped) and tensor infos of a v2/v3 file. */
typedef struct moeb_gguf moeb_gguf;
typedef struct moeb_gguf_tensor {
    int32_t  type;       /* ggml type id */
    int32_t  n_dims;
    int64_t  ne[4];      /* trailing 1s */
    uint64_t offset;     /* absolute byte offset of the data in the file */
    uint64_t nbytes;
} moeb_gguf_tensor;
moeb_gguf *moeb_gguf_open(const char *path);              /* NULL on error (moeb_last_error) */
void       moeb_gguf_close(moeb_gguf *g);
int        moeb_gguf_find_tensor(const moeb_gguf *g, const char *name, moeb_gguf_tensor *out);
int        moeb_gguf_get_u32(const moeb_gguf *g, const char *key, uint32_t *out);
int        moeb_gguf_get_f32(const moeb_gguf *g, const char *key, float *out);
int        moeb_gguf_get_str(const moeb_gguf *g, const char *key, char *out, size_t cap);

/* Copies nbytes of a file from `offset` to device memory `dst`: eight reader threads, each with two
 * 8 MiB pinned staging buffers (128 MiB, allocated on the first load and kept for the process)
 * and its own copy stream, ordered after the work already on `stream`. Loads from several host
 * threads run one at a time. Returns the bytes copied or a negative MOEB_E* code. */
int64_t moeb_load_file_range(const char *path, uint64_t offset, uint64_t nbytes, void *dst, void *stream);

/* Copies the store pages (layer, kind, is_scale, experts[i]) to dst + i * dst_stride, i < n: the
 * hot pool's slots in slot order (kind 0 gate_up, 1 down; is_scale 1: the per-expert down scale,
 * stride 4), with the staging of moeb_load_file_range (pages of at most 8 MiB). verify != 0
 * re-checks each page's checksum. Returns the bytes copied or a negative MOEB_E* code (a missing
 * page, or one longer than dst_stride or 8 MiB: MOEB_EINVAL). */
struct moert_store_reader;
int64_t moeb_load_store_pages(struct moert_store_reader *r, int32_t layer, int32_t kind, int32_t is_scale,
                              const int32_t *experts, int32_t n, void *dst, uint64_t dst_stride, int32_t verify,
                              void *stream);

#ifdef __cplusplus
}
#endif
#endif
