// Host side of libmoeb200.so: the C-ABI entry points declared in include/moeb200.h and the
// moert island ABI of include/moert_cuda.h. Validates arguments, carves workspaces, keeps the
// per-device state (format tables, GELU table, SM count) and launches the sm_100a kernels.
// There is no CPU fallback: without a compute-capability-10 device every compute entry returns
// MOEB_ENODEV (moert_ffn_moe, whose ABI returns nothing, prints and aborts like the reference).
#include "moeb200.h"
#include "moert_cuda.h"
#include "params.h"

#include <cuda_runtime.h>
#include <immintrin.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

using namespace moeb;

namespace {

thread_local std::string g_msg;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_msg = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(MOEB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------- per-device state
constexpr int kMaxDevices = 64;
struct DeviceState {
    bool ready = false;
    int n_sms = 0;
};
std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// ggml-cpu's GELU table (ggml-cpu.c:3784-3793): f16(gelu_tanh(f32(h))) for every f16 bit pattern,
// with gelu_tanh evaluated in ggml's operation order (ggml-cpu/vec.h:963-970). This file is built
// with -ffp-contract=off and the conversions are the F16C instructions ggml uses on x86.
void make_gelu_table(std::vector<uint16_t> &t) {
    t.resize(1u << 16);
    const float c = 0.79788456080286535587989211986876f, a = 0.044715f;
    for (uint32_t h = 0; h < (1u << 16); ++h) {
        const float x = _cvtsh_ss((unsigned short)h);
        const float g = 0.5f * x * (1.0f + tanhf(c * x * (1.0f + a * x * x)));
        t[h] = _cvtss_sh(g, 0);
    }
}

// Makes the current device ready (tables uploaded); returns MOEB_OK or an error code.
int ensure_device(int *n_sms_out = nullptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(MOEB_ENODEV, "no CUDA device: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(MOEB_ENODEV, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState &st = g_dev[dev];
    if (!st.ready) {
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
        if (prop.major != 10)
            return fail(MOEB_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a only", dev, prop.major,
                        prop.minor);
        std::vector<uint16_t> tab;
        make_gelu_table(tab);
        e = upload_gelu_table(tab.data(), 0);
        if (e == cudaSuccess) e = cudaStreamSynchronize(0);
        if (e != cudaSuccess) return cuda_fail(e, "GELU table upload");
        st.n_sms = prop.multiProcessorCount;
        st.ready = true;
    }
    if (n_sms_out) *n_sms_out = st.n_sms;
    return MOEB_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int check_pool(const moeb_pool &pl, int d_model, int n_ff, const char *name) {
    if (pl.n <= 0) return MOEB_OK;
    if (pl.type_gu != MOEB_T_Q4_K && pl.type_gu != MOEB_T_IQ2_S && pl.type_gu != MOEB_T_IQ2_XXS)
        return fail(MOEB_ETYPE, "%s pool: gate_up type %d unsupported (Q4_K=12, IQ2_S=22, IQ2_XXS=16)", name, pl.type_gu);
    if (pl.type_down != MOEB_T_Q5_0 && pl.type_down != MOEB_T_IQ4_NL)
        return fail(MOEB_ETYPE, "%s pool: down type %d unsupported (Q5_0=6, IQ4_NL=20)", name, pl.type_down);
    if (!pl.w_gu || !pl.w_down) return fail(MOEB_EINVAL, "%s pool: null weight pointer", name);
    if (!aligned16(pl.w_gu) || !aligned16(pl.w_down))
        return fail(MOEB_EINVAL, "%s pool: weight bases must be 16-byte aligned", name);
    if ((2LL * n_ff * row_bytes(pl.type_gu, d_model)) % 16 || ((long long)d_model * row_bytes(pl.type_down, n_ff)) % 16)
        return fail(MOEB_EINVAL, "%s pool: expert stride is not a multiple of 16 bytes", name);
    return MOEB_OK;
}

bool prefill_shape_ok(const moeb_layer *L);

// The fused decode kernel keeps a stage ring of whole weight rows and the chunk's activations in
// shared memory; wider layers (the dense MLP's 2112-wide inner dimension) run every batch size on
// the prefill kernels instead.
bool fused_fits(const moeb_layer *L) { return fused_smem_bytes(L->d_model, L->n_ff) <= 227 * 1024; }

int check_layer(const moeb_layer *L) {
    if (!L) return fail(MOEB_EINVAL, "null layer");
    if (L->d_model <= 0 || L->d_model % QK_K) return fail(MOEB_EINVAL, "d_model %d must be a multiple of 256", L->d_model);
    if (L->n_ff <= 0 || L->n_ff % 32) return fail(MOEB_EINVAL, "n_ff %d must be a multiple of 32", L->n_ff);
    if (L->n_expert <= 0 || L->n_expert % 32 || L->n_expert > kMaxE)
        return fail(MOEB_EINVAL, "n_expert %d must be a multiple of 32 and <= %d", L->n_expert, kMaxE);
    if (L->top_k <= 0 || L->top_k > kMaxTopK || L->top_k > L->n_expert)
        return fail(MOEB_EINVAL, "top_k %d out of range (1..%d)", L->top_k, kMaxTopK);
    if (!L->w_router) return fail(MOEB_EINVAL, "null router weights");
    if (L->hot.n > 0 && (!L->exp_slot || !L->slot_exp || !L->slot_state))
        return fail(MOEB_EINVAL, "hot pool given without the residency mirror (exp_slot/slot_exp/slot_state)");
    if (L->hot.n <= 0 && L->cold.n <= 0) return fail(MOEB_EINVAL, "no expert pool");
    if (L->cold.n > 0 && L->cold.n < L->n_expert)
        return fail(MOEB_EINVAL, "cold pool holds %d experts, layer has %d", L->cold.n, L->n_expert);
    if (!fused_fits(L) && !prefill_shape_ok(L))
        return fail(MOEB_EINVAL, "layer shape d_model=%d n_ff=%d: the decode kernel needs more shared memory than an SM "
                                 "has and the prefill kernels do not cover it", L->d_model, L->n_ff);
    int rc = check_pool(L->hot, L->d_model, L->n_ff, "hot");
    if (rc) return rc;
    return check_pool(L->cold, L->d_model, L->n_ff, "cold");
}

// workspace carve for one chunk of up to kFusedTokens tokens
struct LayerWs {
    float *logits;
    uint8_t *xq;
    float *h, *y;
    int32_t *ids, *cnt, *off, *perm;
    float *w;
    uint8_t *qa;
    uint32_t *sync;
    double *nsum;
    size_t bytes;
};

LayerWs carve(const moeb_layer *L, int T, uint8_t *base) {
    LayerWs w{};
    const int P = T * L->top_k;
    size_t o = 0;
    auto take = [&](size_t n) { size_t at = o; o = align_up(o + n, 256); return base ? base + at : nullptr; };
    w.logits = (float *)take(sizeof(float) * T * L->n_expert);
    w.xq = take((size_t)T * xq_stride_bytes(L->d_model));
    w.h = (float *)take(sizeof(float) * 4 * P * 2 * L->n_ff);   // four partial-sum parts
    w.y = (float *)take(sizeof(float) * P * L->d_model);
    w.ids = (int32_t *)take(sizeof(int32_t) * P);
    w.w = (float *)take(sizeof(float) * P);
    w.cnt = (int32_t *)take(sizeof(int32_t) * L->n_expert);
    w.off = (int32_t *)take(sizeof(int32_t) * (L->n_expert + 1));
    w.perm = (int32_t *)take(sizeof(int32_t) * P);
    w.qa = take((size_t)P * fused_qa_stride(L->n_ff));
    w.sync = (uint32_t *)take(sizeof(uint32_t) * fused_sync_words(T, L->d_model, L->n_ff));
    w.nsum = (double *)take(sizeof(double) * T * ((L->d_model + 63) / 64));
    w.bytes = o;
    return w;
}

// prefill path workspace (whole call at once)
struct PrefillWs {
    float *logits, *rpart, *w, *xd, *ad, *y, *nscale;
    int32_t *ids, *cnt, *off, *perm, *pos, *n_tiles;
    PfTile *tiles;
    int8_t *xq8;
    int16_t *xbs;
    uint8_t *bimg, *dimg;
    float *dxt, *hbuf;
    uint32_t *bst;
    int max_tiles;
    size_t bytes;
};

PrefillWs carve_prefill(const moeb_layer *L, int T, uint8_t *base) {
    PrefillWs w{};
    const size_t P = (size_t)T * L->top_k, E = L->n_expert, d = L->d_model, nff = L->n_ff, nsb = d / QK_K;
    size_t o = 0;
    auto take = [&](size_t n) { size_t at = o; o = align_up(o + n, 256); return base ? base + at : nullptr; };
    w.logits = (float *)take(sizeof(float) * T * E);
    w.rpart = (float *)take(sizeof(float) * router_splits(T, (int)E, (int)d) * T * E);
    w.ids = (int32_t *)take(sizeof(int32_t) * P);
    w.w = (float *)take(sizeof(float) * P);
    w.cnt = (int32_t *)take(sizeof(int32_t) * E);
    w.off = (int32_t *)take(sizeof(int32_t) * (E + 1));
    w.perm = (int32_t *)take(sizeof(int32_t) * P);
    w.pos = (int32_t *)take(sizeof(int32_t) * P);
    w.n_tiles = (int32_t *)take(16);
    w.max_tiles = prefill_max_tiles((int)P, (int)E);
    w.tiles = (PfTile *)take(sizeof(PfTile) * w.max_tiles);
    w.xq8 = (int8_t *)take((size_t)T * d);
    w.xd = (float *)take(sizeof(float) * T * nsb);
    w.xbs = (int16_t *)take(sizeof(int16_t) * T * nsb * 16);
    const size_t mt = (size_t)w.max_tiles;
    // the tcgen05 path's gate_up images, or the mid-size path's operand images
    const size_t pf_img = mt * lx_tile_bytes((int)nsb), md_img = md_image_bytes((int)P, (int)E, (int)d, (int)nff);
    w.bimg = (uint8_t *)take(pf_img > md_img ? pf_img : md_img);
    w.dxt = (float *)take(sizeof(float) * mt * nsb * kPrefillTile);
    w.bst = (uint32_t *)take(sizeof(uint32_t) * 8 * mt * nsb * kPrefillTile);
    w.hbuf = (float *)take(sizeof(float) * P * 2 * nff);
    w.dimg = (uint8_t *)take(mt * (nff / 64) * 2 * kPfDnImageBytes);
    w.y = (float *)take(sizeof(float) * P * d);
    w.nscale = (float *)take(sizeof(float) * T);
    w.bytes = o;
    return w;
}

// Batches of at least this many tokens take the prefill path (when the shape allows it).
std::atomic<int32_t> g_prefill_min{64};

bool prefill_shape_ok(const moeb_layer *L) {
    return L->n_ff % 64 == 0 && L->d_model % 128 == 0 && L->d_model / QK_K <= kPrefillMaxSb &&
           L->n_ff / 32 <= kPrefillMaxBlk;
}

bool use_prefill(const moeb_layer *L, int32_t n_tokens) {
    return prefill_shape_ok(L) && (n_tokens >= g_prefill_min.load() || !fused_fits(L));
}

// Prefill-path batches with fewer routed pairs per expert than these run a projection on the
// mid-size kernels (gate_up, down). gate_up: off by default (1) -- the lane-exact tcgen05 kernel
// reproduces the reference's float order, the mid-size kernel only its integer sums; down: the
// down kernel re-streams a tile's weight rows once per 4-block chunk, which loses to the tcgen05
// down on skewed routing already at 16 (one stack layer: 178 vs 152 us).
std::atomic<int32_t> g_mid_max[2] = {{1}, {16}};

bool use_mid(const moeb_layer *L, int32_t n_rows, int kind) {
    const long long P = (long long)n_rows * L->top_k;
    const int32_t m = g_mid_max[kind].load();   // 1: off
    return m > 1 && P < (long long)m * L->n_expert && mid_shape_ok(kind, L->d_model, L->n_ff, (int)P, L->n_expert);
}

PoolView pool_view(const moeb_pool &pl, bool gate_up) {
    PoolView v{};
    v.w = (const uint8_t *)(gate_up ? pl.w_gu : pl.w_down);
    v.type = gate_up ? pl.type_gu : pl.type_down;
    v.n = pl.n;
    v.scale = gate_up ? nullptr : pl.s_down;
    v.ptrs = nullptr;
    return v;
}

}  // namespace

int moeb::set_last_error(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_msg = buf;
    return code;
}

// ================================================================= moeb200.h
extern "C" int moeb_init(void) { return ensure_device(); }

extern "C" const char *moeb_last_error(void) { return g_msg.c_str(); }

extern "C" const char *moeb_version(void) { return "moeb200 0.1 (sm_100a)"; }

extern "C" int32_t moeb_device_error(void *stream) {
    int32_t v = 0;
    if (ensure_device() != MOEB_OK) return MOEB_ENODEV;
    cudaError_t e = read_and_clear_error(&v, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "read device error word");
    return v;
}

size_t moeb::chunk_workspace_size(const moeb_layer *L, int32_t n_tokens) {
    if (!L || n_tokens <= 0) return 0;
    const int T = n_tokens < kFusedTokens ? n_tokens : kFusedTokens;
    return carve(L, T, nullptr).bytes;
}

extern "C" size_t moeb_layer_workspace_size(const moeb_layer *L, int32_t n_tokens) {
    if (!L || n_tokens <= 0) return 0;
    if (use_prefill(L, n_tokens)) return carve_prefill(L, n_tokens, nullptr).bytes;
    return chunk_workspace_size(L, n_tokens);
}

extern "C" int32_t moeb_layer_path(const moeb_layer *L, int32_t n_tokens) {
    const int rc = check_layer(L);
    if (rc) return rc;
    return use_prefill(L, n_tokens) ? 1 : 0;
}

extern "C" int moeb_prefill_profile(int32_t enable) {
    prefill_profile_enable(enable != 0);
    return MOEB_OK;
}

extern "C" int moeb_prefill_profile_read(float *ms, int32_t n) {
    if (!ms || n <= 0) return fail(MOEB_EINVAL, "moeb_prefill_profile_read: null or empty output");
    if (prefill_profile_read(ms, n) != 0)
        return fail(MOEB_EINVAL, "no profiled prefill call on this device (moeb_prefill_profile(1) first)");
    return MOEB_OK;
}

extern "C" int32_t moeb_set_mid_max_pairs(int32_t pairs_per_expert) {
    const int32_t prev = g_mid_max[0].load();
    if (pairs_per_expert > 0) g_mid_max[0].store(pairs_per_expert);
    return prev;
}

extern "C" int32_t moeb_set_mid_max_pairs_down(int32_t pairs_per_expert) {
    const int32_t prev = g_mid_max[1].load();
    if (pairs_per_expert > 0) g_mid_max[1].store(pairs_per_expert);
    return prev;
}

extern "C" int32_t moeb_set_prefill_min_tokens(int32_t n_tokens) {
    const int32_t prev = g_prefill_min.load();
    if (n_tokens > 0) g_prefill_min.store(n_tokens);
    return prev;
}

static int forward_chunks(const moeb_layer *L, const float *x, int32_t n_tokens, float *out,
                          const moeb_layer_aux *aux, void *workspace, cudaStream_t s, int n_sms,
                          const NormArgs &nrm = NormArgs{});

// argument checks shared by both paths of the layer forward
static int check_forward(const moeb_layer *L, const float *x, int32_t n_tokens, float *out, void *workspace,
                         size_t workspace_bytes, size_t need, int *n_sms) {
    int rc = check_layer(L);
    if (rc) return rc;
    if (n_tokens < 0) return fail(MOEB_EINVAL, "n_tokens %d < 0", n_tokens);
    if (n_tokens == 0) return MOEB_OK;
    if (!x || !out) return fail(MOEB_EINVAL, "null x / out");
    if (!aligned16(x) || !aligned16(out) || !aligned16(L->w_router))
        return fail(MOEB_EINVAL, "x, out and router weights must be 16-byte aligned");
    rc = ensure_device(n_sms);
    if (rc) return rc;
    if (!workspace || workspace_bytes < need)
        return fail(MOEB_ESPACE, "workspace of %zu bytes, %zu needed", workspace_bytes, need);
    if (!aligned16(workspace)) return fail(MOEB_EINVAL, "workspace must be 16-byte aligned");
    return MOEB_OK;
}

// The prefill path: nine PDL-chained kernels, the expert matmuls on tcgen05 tensor cores.
static int forward_prefill(const moeb_layer *L, const float *x, int32_t T, float *out, const moeb_layer_aux *aux,
                           void *workspace, cudaStream_t s, int n_sms, const NormArgs &nrm = NormArgs{}) {
    const int d = L->d_model, k = L->top_k, E = L->n_expert, P = T * k;
    PrefillWs w = carve_prefill(L, T, (uint8_t *)workspace);
    PrefillArgs a{};
    a.w_router = L->w_router;
    a.b_router = L->b_router;
    a.x = x;
    a.nrm = nrm;
    a.nscale = w.nscale;
    a.T = T; a.E = E; a.d = d; a.k = k; a.nff = L->n_ff;
    a.res = {L->hot.n, L->exp_slot, L->slot_exp, L->slot_state};
    a.hot_gu = pool_view(L->hot, true);
    a.cold_gu = pool_view(L->cold, true);
    a.hot_dn = pool_view(L->hot, false);
    a.cold_dn = pool_view(L->cold, false);
    a.logits = w.logits; a.rpart = w.rpart; a.ids = w.ids; a.w = w.w;
    a.cnt = w.cnt; a.off = w.off; a.perm = w.perm; a.pos = w.pos;
    a.tiles = w.tiles; a.n_tiles = w.n_tiles;
    a.xq8 = w.xq8; a.xd = w.xd; a.xbs = w.xbs;
    a.bimg = w.bimg; a.dxt = w.dxt; a.bst = w.bst; a.hbuf = w.hbuf; a.dimg = w.dimg; a.max_tiles = w.max_tiles;
    a.h = aux ? aux->gate_up : nullptr;
    a.y = w.y;
    a.out = out;
    a.y_pairs = aux ? aux->down : nullptr;
    a.mid_gu = use_mid(L, T, 0) ? 1 : 0;
    a.mid_dn = use_mid(L, T, 1) ? 1 : 0;
    a.md_max_cb = P / 8 + w.max_tiles;
    cudaError_t e = launch_prefill(a, s, n_sms);
    if (e != cudaSuccess) return MOEB_ECUDA;   // launch_prefill recorded the failing kernel
    if (aux) {
        struct Cp { void *dst; const void *src; size_t n; } cps[] = {
            {aux->logits, w.logits, sizeof(float) * T * E},
            {aux->ids, w.ids, sizeof(int32_t) * P},
            {aux->weights, w.w, sizeof(float) * P},
            {aux->counts, w.cnt, sizeof(int32_t) * E},
            {aux->offsets, w.off, sizeof(int32_t) * (E + 1)},
            {aux->perm, w.perm, sizeof(int32_t) * P},
        };
        for (auto &c : cps) {
            if (!c.dst) continue;
            e = cudaMemcpyAsync(c.dst, c.src, c.n, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "aux copy");
        }
    }
    return MOEB_OK;
}

extern "C" size_t moeb_route_workspace_size(const moeb_layer *L, int32_t n_tokens) {
    if (!L || n_tokens <= 0) return 0;
    return sizeof(float) * 4 * (size_t)n_tokens * L->n_expert;
}

extern "C" int moeb_layer_route(const moeb_layer *L, const float *x, int32_t n_tokens, float *logits, int32_t *ids,
                                float *weights, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_layer(L);
    if (rc) return rc;
    if (n_tokens < 0) return fail(MOEB_EINVAL, "n_tokens %d < 0", n_tokens);
    if (n_tokens == 0) return MOEB_OK;
    if (!x || !logits || !ids || !weights) return fail(MOEB_EINVAL, "moeb_layer_route: null x / logits / ids / weights");
    if (!aligned16(x) || !aligned16(L->w_router)) return fail(MOEB_EINVAL, "x and router weights must be 16-byte aligned");
    rc = ensure_device();
    if (rc) return rc;
    float *part = nullptr;
    if (workspace) {
        if (workspace_bytes < moeb_route_workspace_size(L, n_tokens) || !aligned16(workspace))
            return fail(MOEB_ESPACE, "moeb_layer_route: workspace of %zu bytes (16-byte aligned) < %zu", workspace_bytes,
                        moeb_route_workspace_size(L, n_tokens));
        if (L->d_model % 128) return fail(MOEB_EINVAL, "moeb_layer_route: a split router needs d_model %% 128 == 0");
        part = (float *)workspace;
    }
    cudaError_t e = launch_route(L->w_router, L->b_router, x, n_tokens, L->n_expert, L->d_model, L->top_k, part, logits,
                                 ids, weights, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "route launch");
    return MOEB_OK;
}

extern "C" size_t moeb_routed_workspace_size(const moeb_layer *L, int32_t n_rows) {
    if (!L || n_rows <= 0) return 0;
    return carve_prefill(L, n_rows, nullptr).bytes;
}

static int forward_routed(const moeb_layer *L, const float *x, const uint8_t *xq_rows, int32_t n_rows,
                          const int32_t *ids, const float *weights, float *out, void *workspace, size_t workspace_bytes,
                          void *stream) {
    int n_sms = 0;
    // x or the Q8_K rows, whichever is given, stands for the input in the shared checks
    const float *xin = x ? x : reinterpret_cast<const float *>(xq_rows);
    int rc = check_forward(L, xin, n_rows, out, workspace, workspace_bytes, L ? moeb_routed_workspace_size(L, n_rows) : 0,
                           &n_sms);
    if (rc || n_rows == 0) return rc;
    if (!prefill_shape_ok(L))
        return fail(MOEB_EINVAL, "moeb_layer_forward_routed: n_ff must be a multiple of 64, d_model of 128, d_model <= "
                                 "4096 and n_ff <= %d", kPrefillMaxBlk * 32);
    if (!ids || !weights) return fail(MOEB_EINVAL, "moeb_layer_forward_routed: null ids / weights");
    const int d = L->d_model, k = L->top_k, E = L->n_expert;
    PrefillWs w = carve_prefill(L, n_rows, (uint8_t *)workspace);
    PrefillArgs a{};
    a.w_router = L->w_router;
    a.b_router = L->b_router;
    a.x = x;
    a.T = n_rows; a.E = E; a.d = d; a.k = k; a.nff = L->n_ff;
    a.res = {L->hot.n, L->exp_slot, L->slot_exp, L->slot_state};
    a.hot_gu = pool_view(L->hot, true);
    a.cold_gu = pool_view(L->cold, true);
    a.hot_dn = pool_view(L->hot, false);
    a.cold_dn = pool_view(L->cold, false);
    a.logits = w.logits;
    a.ids = const_cast<int32_t *>(ids);       // read only when routed
    a.w = const_cast<float *>(weights);
    a.cnt = w.cnt; a.off = w.off; a.perm = w.perm; a.pos = w.pos;
    a.tiles = w.tiles; a.n_tiles = w.n_tiles;
    a.xq8 = w.xq8; a.xd = w.xd; a.xbs = w.xbs;
    a.bimg = w.bimg; a.dxt = w.dxt; a.bst = w.bst; a.hbuf = w.hbuf; a.dimg = w.dimg; a.max_tiles = w.max_tiles;
    a.y = w.y;
    a.out = out;
    a.routed = 1;
    a.xq_rows = xq_rows;
    a.mid_gu = use_mid(L, n_rows, 0) ? 1 : 0;
    a.mid_dn = use_mid(L, n_rows, 1) ? 1 : 0;
    a.md_max_cb = n_rows * k / 8 + w.max_tiles;
    cudaError_t e = launch_prefill(a, (cudaStream_t)stream, n_sms);
    if (e != cudaSuccess) return MOEB_ECUDA;
    return MOEB_OK;
}

extern "C" int moeb_layer_forward_routed(const moeb_layer *L, const float *x, int32_t n_rows, const int32_t *ids,
                                         const float *weights, float *out, void *workspace, size_t workspace_bytes,
                                         void *stream) {
    return forward_routed(L, x, nullptr, n_rows, ids, weights, out, workspace, workspace_bytes, stream);
}

extern "C" int moeb_layer_forward_routed_q8k(const moeb_layer *L, const void *xq, int32_t n_rows, const int32_t *ids,
                                             const float *weights, float *out, void *workspace, size_t workspace_bytes,
                                             void *stream) {
    if (n_rows > 0 && !xq) return fail(MOEB_EINVAL, "moeb_layer_forward_routed_q8k: null Q8_K rows");
    return forward_routed(L, nullptr, (const uint8_t *)xq, n_rows, ids, weights, out, workspace, workspace_bytes, stream);
}

extern "C" int moeb_layer_forward(const moeb_layer *L, const float *x, int32_t n_tokens, float *out,
                                  const moeb_layer_aux *aux, void *workspace, size_t workspace_bytes, void *stream) {
    int n_sms = 0;
    int rc = check_forward(L, x, n_tokens, out, workspace, workspace_bytes,
                           L ? moeb_layer_workspace_size(L, n_tokens) : 0, &n_sms);
    if (rc || n_tokens == 0) return rc;
    if (use_prefill(L, n_tokens))
        return forward_prefill(L, x, n_tokens, out, aux, workspace, (cudaStream_t)stream, n_sms);
    return forward_chunks(L, x, n_tokens, out, aux, workspace, (cudaStream_t)stream, n_sms);
}

extern "C" int moeb_layer_forward_gemma4(const moeb_layer *L, const moeb_norms *norms, const float *x,
                                         int32_t n_tokens, float *out, const moeb_layer_aux *aux, void *workspace,
                                         size_t workspace_bytes, void *stream) {
    int n_sms = 0;
    int rc = check_forward(L, x, n_tokens, out, workspace, workspace_bytes,
                           L ? moeb_layer_workspace_size(L, n_tokens) : 0, &n_sms);
    if (rc || n_tokens == 0) return rc;
    if (!norms || !norms->pre_norm || !norms->router_scale || !norms->post_norm)
        return fail(MOEB_EINVAL, "moeb_layer_forward_gemma4: null norms / pre_norm / router_scale / post_norm");
    if (!aligned16(norms->pre_norm) || !aligned16(norms->router_scale) || !aligned16(norms->post_norm))
        return fail(MOEB_EINVAL, "moeb_layer_forward_gemma4: norm vectors must be 16-byte aligned");
    if (!(norms->eps >= 0.f)) return fail(MOEB_EINVAL, "moeb_layer_forward_gemma4: eps must be >= 0");
    if (L->d_model > 4096) return fail(MOEB_EINVAL, "moeb_layer_forward_gemma4: d_model %d > 4096", L->d_model);
    const NormArgs nrm = {norms->pre_norm, norms->router_scale, norms->post_norm, norms->eps};
    if (use_prefill(L, n_tokens))
        return forward_prefill(L, x, n_tokens, out, aux, workspace, (cudaStream_t)stream, n_sms, nrm);
    return forward_chunks(L, x, n_tokens, out, aux, workspace, (cudaStream_t)stream, n_sms, nrm);
}

extern "C" int moeb_rms_norm(const float *x, int32_t rows, int32_t d, const float *w, float scale, float eps,
                             float *out, void *stream) {
    if (rows < 0 || d <= 0 || d % 4) return fail(MOEB_EINVAL, "moeb_rms_norm: rows %d / d %d (d a multiple of 4)", rows, d);
    if (rows == 0) return MOEB_OK;
    if (!x || !out || !aligned16(x) || !aligned16(out) || (w && !aligned16(w)))
        return fail(MOEB_EINVAL, "moeb_rms_norm: null or unaligned x / out / w (16-byte alignment)");
    if (!(eps >= 0.f)) return fail(MOEB_EINVAL, "moeb_rms_norm: eps must be >= 0");
    int rc = ensure_device();
    if (rc != MOEB_OK) return rc;
    cudaError_t e = launch_rms_norm(x, rows, d, w, scale, eps, out, (cudaStream_t)stream);
    return e == cudaSuccess ? MOEB_OK : cuda_fail(e, "rms_norm launch");
}

// ---------------------------------------------------------------- the Gemma-4 feed-forward block
namespace {
std::mutex g_block_mu;
cudaEvent_t g_block_ev[64][2];   // fork / join events per device, created on first use
}  // namespace

extern "C" size_t moeb_ffn_block_workspace_size(const moeb_layer *moe, const moeb_layer *mlp, int32_t n_tokens) {
    if (!moe || !mlp || n_tokens <= 0) return 0;
    return align_up(moeb_layer_workspace_size(moe, n_tokens), 256) + align_up(moeb_layer_workspace_size(mlp, n_tokens), 256) +
           align_up((size_t)n_tokens * mlp->d_model * sizeof(float), 256);
}

extern "C" int moeb_ffn_block_gemma4(const moeb_layer *moe, const moeb_norms *moe_norms, const moeb_layer *mlp,
                                     const moeb_norms *mlp_norms, const float *x, int32_t n_tokens, float *out,
                                     void *workspace, size_t workspace_bytes, void *stream, void *side_stream) {
    if (!moe || !mlp) return fail(MOEB_EINVAL, "moeb_ffn_block_gemma4: null moe / mlp layer");
    if (moe->d_model != mlp->d_model)
        return fail(MOEB_EINVAL, "moeb_ffn_block_gemma4: d_model %d (moe) != %d (mlp)", moe->d_model, mlp->d_model);
    if (mlp->top_k != 1 || mlp->hot.n != 1 || mlp->cold.n > 0)
        return fail(MOEB_EINVAL, "moeb_ffn_block_gemma4: the dense MLP must be a one-expert layer (top_k 1, one hot "
                                 "slot, no cold pool)");
    if (n_tokens < 0) return fail(MOEB_EINVAL, "n_tokens %d < 0", n_tokens);
    const size_t need = moeb_ffn_block_workspace_size(moe, mlp, n_tokens);
    if (n_tokens > 0 && (!workspace || workspace_bytes < need || !aligned16(workspace)))
        return fail(MOEB_EINVAL, "moeb_ffn_block_gemma4: workspace of %zu bytes (16-byte aligned) needed, %zu given", need,
                    workspace_bytes);
    int rc = check_layer(moe);
    if (!rc) rc = check_layer(mlp);
    if (rc || n_tokens == 0) return rc;
    int n_sms = 0;
    if ((rc = ensure_device(&n_sms)) != MOEB_OK) return rc;
    const size_t w_moe = align_up(moeb_layer_workspace_size(moe, n_tokens), 256);
    const size_t w_mlp = align_up(moeb_layer_workspace_size(mlp, n_tokens), 256);
    uint8_t *ws = (uint8_t *)workspace;
    float *tmp = (float *)(ws + w_moe + w_mlp);
    cudaStream_t s = (cudaStream_t)stream, s2 = side_stream ? (cudaStream_t)side_stream : s;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail(MOEB_ENODEV, "moeb_ffn_block_gemma4: no usable device");
    std::lock_guard<std::mutex> lk(g_block_mu);   // record -> wait pairs of one call stay together
    if (s2 != s) {
        for (int i = 0; i < 2; ++i)
            if (!g_block_ev[dev][i] && (e = cudaEventCreateWithFlags(&g_block_ev[dev][i], cudaEventDisableTiming)) != cudaSuccess)
                return cuda_fail(e, "create the block's fork / join events");
        if ((e = cudaEventRecord(g_block_ev[dev][0], s)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(s2, g_block_ev[dev][0], 0)) != cudaSuccess)
            return cuda_fail(e, "fork the dense branch onto the side stream");
    }
    // the dense branch on the side stream, the MoE branch on the main stream, then out = moe + mlp
    int rc2 = moeb_layer_forward_gemma4(mlp, mlp_norms, x, n_tokens, tmp, nullptr, ws + w_moe, w_mlp, s2);
    rc = rc2 ? rc2 : moeb_layer_forward_gemma4(moe, moe_norms, x, n_tokens, out, nullptr, ws, w_moe, s);
    if (s2 != s) {
        // joined on every path, so the side stream never runs past the call
        if ((e = cudaEventRecord(g_block_ev[dev][1], s2)) != cudaSuccess ||
            (e = cudaStreamWaitEvent(s, g_block_ev[dev][1], 0)) != cudaSuccess)
            return cuda_fail(e, "join the dense branch");
    }
    if (rc) return rc;
    if ((e = launch_add_f32(out, tmp, (size_t)n_tokens * moe->d_model, n_sms, s)) != cudaSuccess)
        return cuda_fail(e, "add the block's branches");
    return MOEB_OK;
}

int moeb::layer_forward_chunked(const moeb_layer *L, const float *x, int32_t n_tokens, float *out, void *workspace,
                                size_t workspace_bytes, void *stream) {
    int n_sms = 0;
    int rc = check_forward(L, x, n_tokens, out, workspace, workspace_bytes, chunk_workspace_size(L, n_tokens), &n_sms);
    if (rc || n_tokens == 0) return rc;
    if (!fused_fits(L))
        return fail(MOEB_EINVAL, "layer shape d_model=%d n_ff=%d runs on the prefill kernels only (the decode kernel "
                                 "does not fit in shared memory); use moeb_layer_forward", L->d_model, L->n_ff);
    return forward_chunks(L, x, n_tokens, out, nullptr, workspace, (cudaStream_t)stream, n_sms);
}

// The decode path: one fused cooperative kernel per chunk of up to kFusedTokens tokens.
static int forward_chunks(const moeb_layer *L, const float *x, int32_t n_tokens, float *out, const moeb_layer_aux *aux,
                          void *workspace, cudaStream_t s, int n_sms, const NormArgs &nrm) {
    const int d = L->d_model, k = L->top_k, E = L->n_expert;
    const Residency res = {L->hot.n, L->exp_slot, L->slot_exp, L->slot_state};

    // tokens are independent: longer batches run as consecutive chunks of the fused decode kernel
    for (int t0 = 0; t0 < n_tokens; t0 += kFusedTokens) {
        const int T = n_tokens - t0 < kFusedTokens ? n_tokens - t0 : kFusedTokens;
        const int P = T * k;
        LayerWs w = carve(L, T, (uint8_t *)workspace);
        FusedArgs f{};
        f.w_router = L->w_router;
        f.b_router = L->b_router;
        f.x = x + (size_t)t0 * d;
        f.nrm = nrm;
        f.nsum = w.nsum;
        f.T = T;
        f.E = E;
        f.d = d;
        f.k = k;
        f.nff = L->n_ff;
        f.res = res;
        f.hot_gu = pool_view(L->hot, true);
        f.cold_gu = pool_view(L->cold, true);
        f.hot_dn = pool_view(L->hot, false);
        f.cold_dn = pool_view(L->cold, false);
        f.logits = w.logits;
        f.xq = w.xq;
        f.xq_stride = xq_stride_bytes(d);
        f.h = w.h;
        f.y = w.y;
        f.out = out + (size_t)t0 * d;
        f.ids_out = w.ids;
        f.w_out = w.w;
        f.cnt_out = w.cnt;
        f.off_out = w.off;
        f.perm_out = w.perm;
        f.qa = w.qa;
        f.sync = w.sync;
        cudaError_t e = launch_fused(f, s, n_sms);
        if (e != cudaSuccess) return cuda_fail(e, "fused decode layer launch");

        if (aux) {
            struct Cp { void *dst; const void *src; size_t n; } cps[] = {
                {aux->logits ? aux->logits + (size_t)t0 * E : nullptr, w.logits, sizeof(float) * T * E},
                {aux->ids ? aux->ids + (size_t)t0 * k : nullptr, w.ids, sizeof(int32_t) * P},
                {aux->weights ? aux->weights + (size_t)t0 * k : nullptr, w.w, sizeof(float) * P},

                {aux->down ? aux->down + (size_t)t0 * k * d : nullptr, w.y, sizeof(float) * P * d},
            };
            for (auto &c : cps) {
                if (!c.dst) continue;
                e = cudaMemcpyAsync(c.dst, c.src, c.n, cudaMemcpyDeviceToDevice, s);
                if (e != cudaSuccess) return cuda_fail(e, "aux copy");
            }
            if (aux->gate_up) {
                const size_t n = (size_t)P * 2 * L->n_ff;
                e = launch_sum4(w.h, n, aux->gate_up + (size_t)t0 * k * 2 * L->n_ff, n, s);
                if (e != cudaSuccess) return cuda_fail(e, "aux gate_up");
            }
            // the dispatch outputs describe one chunk; they are reported for single-chunk calls
            if (n_tokens <= kFusedTokens) {
                if (aux->counts) e = cudaMemcpyAsync(aux->counts, w.cnt, sizeof(int32_t) * E, cudaMemcpyDeviceToDevice, s);
                if (e == cudaSuccess && aux->offsets)
                    e = cudaMemcpyAsync(aux->offsets, w.off, sizeof(int32_t) * (E + 1), cudaMemcpyDeviceToDevice, s);
                if (e == cudaSuccess && aux->perm)
                    e = cudaMemcpyAsync(aux->perm, w.perm, sizeof(int32_t) * P, cudaMemcpyDeviceToDevice, s);
                if (e != cudaSuccess) return cuda_fail(e, "aux copy");
            }
        }
    }
    return MOEB_OK;
}

extern "C" int moeb_router_topk(const float *logits, int32_t n_tokens, int32_t n_expert, int32_t top_k, int32_t *ids,
                                float *weights, void *stream) {
    if (!logits || n_tokens <= 0 || n_expert <= 0 || n_expert % 32 || n_expert > kMaxE || top_k <= 0 ||
        top_k > kMaxTopK || top_k > n_expert)
        return fail(MOEB_EINVAL, "moeb_router_topk: bad shape T=%d E=%d k=%d", n_tokens, n_expert, top_k);
    int rc = ensure_device();
    if (rc) return rc;
    for (int t0 = 0; t0 < n_tokens; t0 += kMaxDecodeT) {
        const int T = n_tokens - t0 < kMaxDecodeT ? n_tokens - t0 : kMaxDecodeT;
        RouteSrc r = {logits + (size_t)t0 * n_expert, nullptr, 0, T, n_expert, top_k};
        cudaError_t e = launch_route_only(r, ids ? ids + (size_t)t0 * top_k : nullptr,
                                          weights ? weights + (size_t)t0 * top_k : nullptr, nullptr, nullptr, nullptr,
                                          (cudaStream_t)stream);
        if (e != cudaSuccess) return cuda_fail(e, "route launch");
    }
    return MOEB_OK;
}

extern "C" int moeb_dispatch(const int32_t *ids, int32_t n_tokens, int32_t top_k, int32_t n_expert, int32_t *counts,
                             int32_t *offsets, int32_t *perm, void *stream) {
    if (!ids || n_tokens <= 0 || n_tokens > kMaxDecodeT || n_expert <= 0 || n_expert % 32 || n_expert > kMaxE ||
        top_k <= 0 || top_k > kMaxTopK)
        return fail(MOEB_EINVAL, "moeb_dispatch: bad shape T=%d E=%d k=%d (T <= %d on this path)", n_tokens, n_expert,
                    top_k, kMaxDecodeT);
    int rc = ensure_device();
    if (rc) return rc;
    RouteSrc r = {nullptr, ids, top_k, n_tokens, n_expert, top_k};
    cudaError_t e = launch_route_only(r, nullptr, nullptr, counts, offsets, perm, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "dispatch launch");
    return MOEB_OK;
}

extern "C" int moeb_dequantize(int32_t type, const void *src, float *dst, int64_t n_rows, int64_t n_per_row, void *stream) {
    if (type != MOEB_T_Q4_K && type != MOEB_T_IQ2_S && type != MOEB_T_Q5_0 && type != MOEB_T_IQ4_NL &&
        type != MOEB_T_IQ2_XXS && type != MOEB_T_Q8_0)
        return fail(MOEB_ETYPE, "moeb_dequantize: type %d unsupported", type);
    const int blk = (type == MOEB_T_Q4_K || type == MOEB_T_IQ2_S || type == MOEB_T_IQ2_XXS) ? QK_K : QK32;
    if (!src || !dst || n_rows <= 0 || n_per_row <= 0 || n_per_row % blk)
        return fail(MOEB_EINVAL, "moeb_dequantize: bad shape");
    int rc = ensure_device();
    if (rc) return rc;
    cudaError_t e = launch_dequant(type, src, dst, n_rows, n_per_row, (cudaStream_t)stream);
    return e == cudaSuccess ? MOEB_OK : cuda_fail(e, "dequant launch");
}

extern "C" int moeb_quantize_act(int32_t wtype, const float *x, void *dst, int64_t n_rows, int64_t n_per_row,
                                 void *stream) {
    int32_t vdt;
    if (wtype == MOEB_T_Q4_K || wtype == MOEB_T_IQ2_S || wtype == MOEB_T_IQ2_XXS) vdt = T_Q8_K;
    else if (wtype == MOEB_T_Q5_0 || wtype == MOEB_T_IQ4_NL) vdt = T_Q8_0;
    else return fail(MOEB_ETYPE, "moeb_quantize_act: weight type %d unsupported", wtype);
    if (!x || !dst || n_rows <= 0 || n_per_row <= 0 || n_per_row % (vdt == T_Q8_K ? QK_K : QK32))
        return fail(MOEB_EINVAL, "moeb_quantize_act: bad shape");
    int rc = ensure_device();
    if (rc) return rc;
    cudaError_t e = launch_quant_act(vdt, x, dst, n_rows, n_per_row, (cudaStream_t)stream);
    return e == cudaSuccess ? MOEB_OK : cuda_fail(e, "quant launch");
}

extern "C" size_t moeb_row_size(int32_t type, int64_t n_per_row) { return (size_t)row_bytes(type, n_per_row); }

// ================================================================= moert_cuda.h
namespace {

moert_cuda_config g_cfg = {1, 0, 0, 3, 0, 0, 0, 0, 0};

struct Binding {
    const void *w_hot = nullptr, *w_cold = nullptr;
    int32_t hot_type = 0, cold_type = 0, n_hot = 0, n_cold = 0;
    const void *const *hot_table = nullptr;
    int32_t hot_table_n = 0, hot_table_type = 0;
};
constexpr int kMaxLayers = 128;
Binding g_bind[kMaxLayers][2];

struct RouteCounters {
    int32_t *dev = nullptr;
    int32_t nl = 0, ne = 0;
} g_rc;

std::atomic<long long> g_fires{0}, g_op_ns{0};

[[noreturn]] void island_abort(const char *what) {
    fprintf(stderr, "moert_ffn_moe: %s\n", what);
    abort();
}

}  // namespace

extern "C" void moert_cuda_configure(const moert_cuda_config *cfg) {
    if (cfg) g_cfg = *cfg;
}

extern "C" int moeb_bind_pools(int32_t il, int32_t kind, const void *w_hot, int32_t hot_type, int32_t n_hot,
                               const void *w_cold, int32_t cold_type, int32_t n_cold) {
    if (il < 0 || il >= kMaxLayers || kind < 0 || kind > 1) return fail(MOEB_EINVAL, "bind: il/kind out of range");
    Binding &b = g_bind[il][kind];
    b.w_hot = w_hot;
    b.hot_type = hot_type;
    b.n_hot = n_hot;
    b.w_cold = w_cold;
    b.cold_type = cold_type;
    b.n_cold = n_cold;
    return MOEB_OK;
}

extern "C" void moert_ffn_moe(const moert_ffn_moe_args *a, const moert_ffn_moe_host *h) {
    const auto t_start = std::chrono::steady_clock::now();
    if (!a) island_abort("null args");
    if (a->planc_mode != 0) island_abort("only planc_mode 0 (device-resident cold pool) is served on B200");
    if (a->kind != 0 && a->kind != 1) island_abort("kind must be 0 (gate_up) or 1 (down)");
    if (a->il < 0 || a->il >= kMaxLayers) island_abort("layer index out of range");
    int n_sms = 0;
    if (ensure_device(&n_sms) != MOEB_OK) island_abort(g_msg.c_str());
    const Binding &b = g_bind[a->il][a->kind];
    cudaStream_t s = (cudaStream_t)a->stream;
    const int kind = a->kind, k = a->n_used, T = a->n_tokens;
    if (k <= 0 || k > kMaxTopK || T <= 0) island_abort("n_used / n_tokens out of range");
    if (a->n_expert <= 0 || a->n_expert > kMaxE || a->n_expert % 32) island_abort("n_expert must be a multiple of 32, <= 256");
    const int blk = kind == 0 ? QK_K : QK32;
    if (a->d_in % blk || a->d_out % kGroupRows) island_abort("d_in / d_out not supported");

    PoolView hot{}, cold{};
    hot.w = (const uint8_t *)b.w_hot;
    hot.type = b.hot_type;
    hot.n = b.n_hot;
    hot.scale = kind == 1 ? (const float *)a->s_hot : nullptr;
    if (b.hot_table && b.hot_table_n == a->k) { hot.ptrs = b.hot_table; hot.type = b.hot_table_type; }
    cold.w = (const uint8_t *)b.w_cold;
    cold.type = a->cold_type_tag;
    cold.n = a->n_expert;
    cold.scale = kind == 1 ? (const float *)a->s_cold : nullptr;
    if (!cold.w && a->has_w_cold) island_abort("cold pool not bound (moeb_bind_pools)");
    const Residency res = {a->k, (const int32_t *)a->exp_slot, (const int32_t *)a->slot_exp, (const int32_t *)a->slot_state};

    int32_t *rc_counts = nullptr, *rc_hits = nullptr;
    if (g_rc.dev && kind == 0 && a->il < g_rc.nl && a->n_expert == g_rc.ne) {
        rc_counts = g_rc.dev + (size_t)a->il * g_rc.ne;
        rc_hits = g_rc.dev + (size_t)g_rc.nl * g_rc.ne + (size_t)a->il * 2;
    }

    // scratch from the caller's pool (strict LIFO): the Q8_K activations of gate_up
    void *scratch = nullptr;
    const int xs = xq_stride_bytes(a->d_in);
    if (kind == 0) {
        if (!h || !h->pool_alloc) island_abort("gate_up needs the host pool for activation scratch");
        scratch = h->pool_alloc(h->user, (uint64_t)xs * (T < kMaxDecodeT ? T : kMaxDecodeT) + 256);
    }
    const int32_t *ids = (const int32_t *)a->ids;
    const float *cur = (const float *)a->cur;
    float *dst = (float *)a->dst;
    for (int t0 = 0; t0 < T; t0 += kMaxDecodeT) {
        const int Tc = T - t0 < kMaxDecodeT ? T - t0 : kMaxDecodeT;
        GemvParams g{};
        g.route = {nullptr, ids + (size_t)t0 * a->ids_s1, a->ids_s1, Tc, a->n_expert, k};
        g.res = res;
        g.hot = hot;
        g.cold = cold;
        g.d_in = a->d_in;
        g.d_out = a->d_out;
        g.y = dst + (size_t)t0 * k * a->d_out;
        g.rc_counts = rc_counts;
        g.rc_hits = rc_hits;
        cudaError_t e;
        if (kind == 0) {
            // gate_up: one shared activation column per token (cur is [d_in, 1, T])
            e = launch_quant_q8k(cur + (size_t)t0 * a->d_in, (uint8_t *)scratch, Tc, a->d_in, xs, s);
            if (e != cudaSuccess) island_abort(cudaGetErrorString(e));
            g.kind = 0;
            g.xq = (const uint8_t *)scratch;
            g.xq_stride = xs;
        } else {
            // down: one activation column per routed pair (cur is [d_in, n_used, T])
            g.kind = 2;
            g.a = cur + (size_t)t0 * k * a->d_in;
            g.a_per_pair = 1;
            g.apply_scale = 1;
        }
        e = launch_gemv(g, s, false, n_sms);
        if (e != cudaSuccess) island_abort(cudaGetErrorString(e));
    }
    if (scratch) h->pool_free(h->user, scratch);
    g_fires++;
    g_op_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t_start).count();
}

extern "C" int32_t moert_cuda_route_counts_enable(int32_t n_layers, int32_t n_expert) {
    if (n_layers <= 0 || n_expert <= 0) return 0;
    if (ensure_device() != MOEB_OK) return 0;
    if (g_rc.dev) { cudaFree(g_rc.dev); g_rc.dev = nullptr; }
    const size_t n = (size_t)n_layers * n_expert + (size_t)n_layers * 2;
    if (cudaMalloc(&g_rc.dev, n * sizeof(int32_t)) != cudaSuccess) { g_rc.dev = nullptr; return 0; }
    if (cudaMemset(g_rc.dev, 0, n * sizeof(int32_t)) != cudaSuccess) return 0;
    g_rc.nl = n_layers;
    g_rc.ne = n_expert;
    return 1;
}

extern "C" int32_t moert_cuda_route_counts_fetch(int32_t *dst, int32_t reset) {
    if (!g_rc.dev || !dst) return 0;
    const size_t n = (size_t)g_rc.nl * g_rc.ne + (size_t)g_rc.nl * 2;
    if (cudaMemcpy(dst, g_rc.dev, n * sizeof(int32_t), cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    if (reset && cudaMemset(g_rc.dev, 0, n * sizeof(int32_t)) != cudaSuccess) return 0;
    return 1;
}

extern "C" int32_t moert_cuda_host_register_pinned(void *base, uint64_t size) {
    if (!base || !size) return 0;
    cudaError_t e = cudaHostRegister(base, size, cudaHostRegisterDefault);
    if (e == cudaErrorHostMemoryAlreadyRegistered) { cudaGetLastError(); return 1; }
    return e == cudaSuccess ? 1 : (cudaGetLastError(), 0);
}

extern "C" void moert_cuda_host_unregister(void *base) {
    if (base && cudaHostUnregister(base) != cudaSuccess) cudaGetLastError();
}

extern "C" int32_t moert_cuda_host_register_mapped(void *base, uint64_t size) {
    if (!base || !size) return 0;
    cudaError_t e = cudaHostRegister(base, size, cudaHostRegisterMapped);
    if (e == cudaErrorHostMemoryAlreadyRegistered) { cudaGetLastError(); return 1; }
    return e == cudaSuccess ? 1 : (cudaGetLastError(), 0);
}

extern "C" void *moert_cuda_host_map(void *base, uint64_t size) {
    if (!moert_cuda_host_register_mapped(base, size)) return nullptr;
    void *dev = nullptr;
    if (cudaHostGetDevicePointer(&dev, base, 0) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    return dev;
}

extern "C" void moert_cuda_stats_get(moert_cuda_stats *out) {
    if (!out) return;
    memset(out, 0, sizeof *out);
    out->fires = g_fires.load();
    out->op_host_ns = g_op_ns.load();
}

// The transfer director moves experts between host RAM and VRAM slots; on B200 both classes are
// HBM-resident, so the asynchronous transport is refused (0) and callers copy themselves, which
// is the reference contract for a refused copy (cuda.h:248-250).
extern "C" int32_t moert_cuda_dir_init(int32_t, int32_t, int32_t) { return 0; }
extern "C" int32_t moert_cuda_dir_async(void *, const void *, uint64_t) { return 0; }
extern "C" int64_t moert_cuda_dir_mark(void) { return 0; }
extern "C" int64_t moert_cuda_dir_poll(int32_t) { return 0; }
extern "C" void moert_cuda_dir_stats_get(moert_cuda_dir_stats *out) {
    if (out) memset(out, 0, sizeof *out);
}
extern "C" int64_t moert_cuda_dir_gate(int32_t, int64_t) { return 0; }

// Residency publication: n synchronous host -> device copies (cuda.h:258-260).
extern "C" int32_t moert_cuda_publish_h2d(int32_t n, void *const *dsts, const void *const *srcs, const uint64_t *sizes) {
    if (n < 0 || (n > 0 && (!dsts || !srcs || !sizes))) return 0;
    for (int32_t i = 0; i < n; ++i)
        if (cudaMemcpy(dsts[i], srcs[i], sizes[i], cudaMemcpyHostToDevice) != cudaSuccess) return 0;
    return 1;
}

extern "C" void moert_cuda_set_hot_table(int32_t il, int32_t kind, const void *const *dev_ptrs, int32_t n, int32_t type_tag) {
    if (il < 0 || il >= kMaxLayers || kind < 0 || kind > 1) return;
    Binding &b = g_bind[il][kind];
    b.hot_table = n > 0 ? dev_ptrs : nullptr;
    b.hot_table_n = n > 0 ? n : 0;
    b.hot_table_type = type_tag;
}
