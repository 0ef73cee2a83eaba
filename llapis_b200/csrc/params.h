// Kernel parameter blocks, shape helpers and launcher declarations shared by the device
// translation unit (kernels.cu) and the host-side C-ABI (api.cpp). Host-safe: no device code.
#pragma once

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define MOEB_HD __host__ __device__
#else
#define MOEB_HD
#endif

namespace moeb {

// ggml type ids (third_party/llama/ggml/include/ggml.h:390-432); they travel through the moert
// ABI as opaque "type tags".
enum : int32_t {
    T_F32 = 0, T_F16 = 1, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q8_K = 15, T_IQ2_XXS = 16, T_IQ4_NL = 20, T_IQ2_S = 22,
};

constexpr int QK_K = 256;
constexpr int QK32 = 32;
constexpr int B_Q4_K = 144;    // d f16 | dmin f16 | scales[12] | qs[128]
constexpr int B_IQ2_S = 82;    // d f16 | qs[32] | signs[32] | qh[8] | scales[8]
constexpr int B_IQ2_XXS = 66;  // d f16 | 8 x (4 codebook indices u8 | u32: 4 x 7-bit sign index, 4-bit sub-scale)
constexpr int B_Q5_0 = 22;     // d f16 | qh[4] | qs[16]
constexpr int B_IQ4_NL = 18;   // d f16 | qs[16]
constexpr int B_Q8_K = 292;    // d f32 | qs[256] | bsums[16] i16
constexpr int B_Q8_0 = 34;     // d f16 | qs[32]

MOEB_HD inline int64_t row_bytes(int32_t type, int64_t n) {
    switch (type) {
        case T_F32:    return n * 4;
        case T_F16:    return n * 2;
        case T_Q4_K:   return n / QK_K * B_Q4_K;
        case T_IQ2_S:  return n / QK_K * B_IQ2_S;
        case T_IQ2_XXS: return n / QK_K * B_IQ2_XXS;
        case T_Q5_0:   return n / QK32 * B_Q5_0;
        case T_IQ4_NL: return n / QK32 * B_IQ4_NL;
        case T_Q8_K:   return n / QK_K * B_Q8_K;
        case T_Q8_0:   return n / QK32 * B_Q8_0;
        default:       return 0;
    }
}

constexpr int kThreads = 256;            // 8 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kMaxDecodeT = 16;          // tokens per call on the GEMV path
constexpr int kMaxE = 256;               // experts per layer (multiple of 32)
constexpr int kMaxTopK = 16;
constexpr int kMaxPairs = kMaxDecodeT * kMaxTopK;
constexpr int kTokChunk = 4;             // tokens dotted per pass over a decoded weight row
constexpr int kGroupRows = 8;            // work-split granularity (16-byte aligned for all types)

// Residency classes of a routed pair (moert/cuda/ffn_moe.cu:101-104).
struct Residency {
    int32_t n_slots;
    const int32_t *exp_slot, *slot_exp, *slot_state;
};

// One precision class of a projection: pool base, type, rows, and the per-entry down scale.
struct PoolView {
    const uint8_t *w;     // [n][rows][row_bytes]
    int32_t type;
    int32_t n;
    const float *scale;   // [n] or nullptr
    const void *const *ptrs;   // optional device table: entry i at ptrs[i] instead of w + i*stride
};

// Routing source for the in-CTA dispatch: either logits (softmax/top-k in the CTA) or given ids.
struct RouteSrc {
    const float *logits;    // [T][E] or nullptr
    const int32_t *ids;     // [T][ids_s1] or nullptr (when logits == nullptr)
    int32_t ids_s1;
    int32_t T, E, k;
};

// gate_up / down grouped GEMV problem.
struct GemvParams {
    RouteSrc route;
    Residency res;
    PoolView hot, cold;
    int32_t d_in, d_out;
    // activations
    const uint8_t *xq;       // gate_up: Q8_K rows [T][xq_stride] (per token)
    int32_t xq_stride;
    const float *h;          // down (from_h): f32 [P][2*d_in] gate_up outputs -> GeGLU -> Q8_0
    const float *a;          // down (plain): f32 [P][d_in] activations (or [n_cols][d_in] with a_per_pair=0)
    int32_t a_per_pair;
    int32_t kind;            // 0 gate_up (Q8_K from xq), 1 down from h, 2 down from a
    float *y;                // [P][d_out]
    int32_t apply_scale;
    // routing outputs for inspection (written by CTA 0 when non-null)
    int32_t *ids_out;
    float *w_out;
    int32_t *cnt_out, *off_out, *perm_out;
    // device routing counters (moert_cuda_route_counts_*): [E] routed pairs, [2] hot/cold pairs
    int32_t *rc_counts, *rc_hits;
};

// The norms around the Gemma-4 MoE block (gemma4.cpp:394-427), device pointers to f32 [d]:
//   expert input  = rms_norm(x) * pre            (ffn_pre_norm_2)
//   router input  = rms_norm(x) / sqrt(d) * router  (ffn_gate_inp_s)
//   output        = rms_norm(moe) * post         (ffn_post_norm_2)
// pre == nullptr: the plain layer (x feeds both the router and the experts, no output norm).
struct NormArgs {
    const float *pre, *router, *post;
    float eps;
};

// the fused decode layer (one cooperative launch per chunk of <= kFusedTokens tokens)
constexpr int kFusedTokens = 8;
struct FusedArgs {
    const float *w_router, *b_router, *x;
    int32_t T, E, d, k, nff;
    NormArgs nrm;
    double *nsum;            // [kFusedTokens][ceil(d / 64)] output sums of squares per 64-row block (norms only)
    Residency res;
    PoolView hot_gu, cold_gu, hot_dn, cold_dn;
    float *logits;
    uint8_t *xq;
    int32_t xq_stride;
    float *h, *y, *out;         // h: four [T*k][2 nff] partial-sum parts of gate_up
    int32_t *ids_out, *cnt_out, *off_out, *perm_out;
    float *w_out;
    uint8_t *qa;             // [T*k][q80 row of n_ff] down activations (Q8_0), expert-sorted slot order
    uint32_t *sync;          // fused_sync_words(T, d, nff) zero-initialised-by-the-kernel counters
};
// counters: gate_up rows per (unique expert, 32-row ff block), finished blocks per unique expert,
// down rows per (token, 64-row output block), combined output blocks per token
MOEB_HD inline int fused_sync_words(int T, int d, int nff) {
    return kFusedTokens * kMaxTopK * (nff / 32 + 1) + T * ((d + 63) / 64) + T;
}

// the prefill path (tcgen05 grouped GEMMs; prefill.cuh)
constexpr int kPrefillTile = 128;        // routed pairs per expert tile (MMA N)
constexpr int kPrefillMaxSb = 16;        // d_model <= 4096
constexpr int kPrefillMaxBlk = 128;      // n_ff <= 4096
// One expert tile: up to kPrefillTile consecutive slots of the expert-sorted pair order.
struct PfTile {
    int32_t cls;     // 0 hot pool, 1 cold pool
    int32_t widx;    // entry of that pool (slot or expert)
    int32_t slot0;   // first slot
    int32_t n;       // pairs
};
MOEB_HD inline int prefill_max_tiles(int P, int E) { return P / kPrefillTile + E + 1; }
// fp16 operand images of one tile in the tensor cores' canonical layout (16 bytes per core row).
// gate_up (gateup_lx.cuh): per tile, pass (0..3) and super-block one image of 16 row groups x 8
// cores x 128 B, pass-major; down: 128 rows x 8 core columns (two 32-blocks) per stage
constexpr int kLxImgMain = (kPrefillTile / 8) * 8 * 128;
MOEB_HD inline size_t lx_tile_bytes(int nsb) { return (size_t)nsb * 4 * kLxImgMain; }
MOEB_HD inline size_t lx_image_off(int nsb, int pass, int sb) { return (size_t)(pass * nsb + sb) * kLxImgMain; }
constexpr int kPfDnImageBytes = kPrefillTile * 8 * 16;
struct PrefillArgs {
    const float *w_router, *b_router, *x;
    int32_t T, E, d, k, nff;
    NormArgs nrm;
    float *nscale;              // [T] rms_norm row scales of x (norms only)
    Residency res;
    PoolView hot_gu, cold_gu, hot_dn, cold_dn;
    float *logits;              // [T][E]
    float *rpart;               // [router_splits][T][E] router partial sums (one per K part)
    int32_t *ids;               // [T][k]
    float *w;                   // [T][k]
    int32_t *cnt, *off;         // [E], [E + 1]
    int32_t *perm, *pos;        // [P] slot -> pair, pair -> slot (-1: expert without a pool)
    PfTile *tiles;              // [prefill_max_tiles]
    int32_t *n_tiles;
    int8_t *xq8;                // [T][d]
    float *xd;                  // [T][d / 256]
    int16_t *xbs;               // [T][d / 256][16]
    uint8_t *bimg;              // [max_tiles][lx_tile_bytes] gate_up B operand images (or the mid path's)
    float *dxt;                 // [max_tiles][d / 256][kPrefillTile] Q8_K scales per tile row
    uint32_t *bst;              // [max_tiles][d / 256][kPrefillTile][8] Q8_K bsums per tile row, fp16 pairs
    float *hbuf;                // [P][2 nff] gate_up outputs, slot order
    uint8_t *dimg;              // [max_tiles][nff / 64][2][kPfDnImageBytes] down B operand images (hi, lo)
    int32_t max_tiles;
    float *h;                   // optional [P][2 nff] gate_up outputs, pair order
    float *y;                   // [P][d] down outputs, slot order
    float *out;                 // [T][d]
    float *y_pairs;             // optional [P][d] down outputs, pair order
    int32_t routed;             // 1: ids / w are given (the router and top-k kernels are skipped)
    const uint8_t *xq_rows;     // routed only, optional: the tokens' Q8_K rows in ggml layout ([T][d / 256]
                                // blocks of d f32 | qs[256] | bsums[16] i16), unpacked in place of quantising x
    int32_t mid_gu, mid_dn;     // 1: that projection runs the mid-size kernels (int8 MMAs on the weight codes;
                                // bimg holds their operand images), 0: the tcgen05 kernels
    int32_t md_max_cb;          // mid path: bound on the column blocks (P / 8 + max_tiles)
};
// K parts of the prefill router GEMM: the smallest divisor s >= 4 of d / 32 (32-wide K chunks) that
// gives at least one wave of 64-token x 128-expert CTAs on 148 SMs, at most d / 128 (four chunks per
// CTA: the top-k kernel adds the parts in order, so more parts cost more there)
MOEB_HD inline int router_splits(int T, int E, int d) {
    const int nch = d / 32, tiles = ((T + 63) / 64) * ((E + 127) / 128);
    int best = 4;
    for (int s = 4; s <= nch / 4; ++s) {
        if (nch % s) continue;
        best = s;
        if (tiles * s >= 148) break;
    }
    return best;
}
// mid path: operand image bytes (one 8-pair column block of gate_up, the larger of the two kinds)
MOEB_HD inline size_t md_image_bytes(int P, int E, int d, int nff) {
    const size_t cb = (size_t)(P / 8 + prefill_max_tiles(P, E));
    const size_t gu = (size_t)(d / 256) * 5 * 512, dn = (size_t)(nff / 32) * 512;
    return cb * (gu > dn ? gu : dn);
}
// router logits + softmax/top-k/weights only (the first two prefill kernels)
cudaError_t launch_route(const float *w_router, const float *b_router, const float *x, int T, int E, int d, int k,
                         float *part, float *logits, int32_t *ids, float *w, cudaStream_t s);
cudaError_t launch_prefill(const PrefillArgs &a, cudaStream_t s, int n_sms);
// whether the mid-size kernel of a projection (0 gate_up, 1 down) covers this shape (shared
// memory, tile and unit counts) for P routed pairs
bool mid_shape_ok(int kind, int d, int nff, int P, int E);
// router, top-k, dispatch, activation quantisation, gather, gate_up, GeGLU, down, combine
constexpr int kPrefillKernels = 9;
void prefill_profile_enable(bool on);
int prefill_profile_read(float *ms, int n);

MOEB_HD inline int xq_stride_bytes(int d) { return (int)(((d / QK_K) * B_Q8_K + 15) / 16 * 16); }
// Q8_0 activation row in shared memory: qs[nb][32] | d[nb] f32 | qsum[nb] i32
MOEB_HD inline int q80_stride(int d_in) { return ((d_in / 32) * 40 + 15) / 16 * 16; }
// rows of the fused kernel's down activations in global memory start on their own 128-byte lines,
// so a row read through L1 never shares a line with a row another CTA is still writing
MOEB_HD inline int fused_qa_stride(int nff) { return (q80_stride(nff) + 127) / 128 * 128; }

// host-side launch helpers (decode.cu); `pdl` chains the launch to the previous kernel in the stream
cudaError_t launch_gemv(const GemvParams &p, cudaStream_t s, bool pdl, int n_sms);
cudaError_t launch_quant_q8k(const float *x, uint8_t *dst, int rows, int d, int stride, cudaStream_t s);
size_t gemv_smem_bytes(int kind, int d_in, int T);
cudaError_t launch_fused(const FusedArgs &a, cudaStream_t s, int n_sms);
// dst[i] = ((h[i] + h[i + stride]) + h[i + 2 stride]) + h[i + 3 stride]: the fused kernel's gate_up
// rows are four partial sums (super-block quarters); this adds them for the aux output
cudaError_t launch_sum4(const float *h, size_t stride, float *dst, size_t n, cudaStream_t s);
cudaError_t launch_add_f32(float *out, const float *a, size_t n, int n_sms, cudaStream_t s);
cudaError_t launch_rms_norm(const float *x, int rows, int d, const float *w, float c, float eps, float *out,
                            cudaStream_t s);
size_t fused_smem_bytes(int d, int nff);
// standalone pieces behind the moeb_* inspection entry points
cudaError_t launch_route_only(const RouteSrc &r, int32_t *ids, float *w, int32_t *cnt, int32_t *off, int32_t *perm,
                              cudaStream_t s);
cudaError_t launch_dequant(int32_t type, const void *src, float *dst, int64_t rows, int64_t n, cudaStream_t s);
cudaError_t launch_quant_act(int32_t vdt, const float *x, void *dst, int64_t rows, int64_t n, cudaStream_t s);
// device state: format tables, GELU table upload, error word
cudaError_t upload_gelu_table(const uint16_t *host_table, cudaStream_t s);
cudaError_t read_and_clear_error(int32_t *out, cudaStream_t s);
// the decode-chunk path of the layer forward with its own (one-chunk) workspace bound; the
// allocation-free entry uses it for every batch size
}  // namespace moeb
struct moeb_layer;
namespace moeb {
size_t chunk_workspace_size(const moeb_layer *L, int32_t n_tokens);
int layer_forward_chunked(const moeb_layer *L, const float *x, int32_t n_tokens, float *out, void *workspace,
                          size_t workspace_bytes, void *stream);
// records the message moeb_last_error() returns; returns `code`
int set_last_error(int code, const char *fmt, ...);

}  // namespace moeb
