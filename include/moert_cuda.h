/*
 * moert_cuda.h — the MoE CUDA island ABI, served by libmoeb200.so.
 *
 * Drop-in replacement for the reference island's device-pointer ABI
 * (moert/include/moert/cuda.h). Every struct below has the same members, order and types as the
 * reference so the ggml trampoline (third_party/llama/ggml/src/ggml-cuda/moe-dual.cu:98-157) and
 * the host shim (src/moe_dual.cpp) link against this library unchanged. Plain C: raw device
 * pointers, the caller's CUDA stream as void*, no ggml or torch types.
 *
 * What changes behind the ABI: both precision classes are HBM-resident on the B200, so
 * moert_ffn_moe runs hot and cold pairs with this library's own sm_100a kernels (the host `mm`
 * vtable entry is not called) and there is no Pmax <= 32 ceiling. The RAM-cold machinery
 * (planc_mode 1/2, CPU sidecar callbacks, the transfer director) is accepted at the ABI but refused
 * at run time: those calls return 0 ("refused, the caller copies itself") exactly as the reference
 * does when a service is unavailable.
 */
#ifndef MOEB200_MOERT_CUDA_H
#define MOEB200_MOERT_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Pair ceiling of the reference's single-warp partition (cuda.h:39). Kept for source
 * compatibility; this implementation accepts any n_used * n_tokens. */
#define MOERT_COLDCPU_GS_PMAX_MAX 32

/* replaces moert/include/moert/cuda.h:41-69 (same layout) */
typedef struct moert_cuda_config {
    int32_t  counted;            /* live-channel guard; always effectively on here          */
    int32_t  copy_stream;        /* RAM-cold copy stream: not used (no RAM-cold tier)        */
    int32_t  coldcpu;            /* CPU cold sidecar: not used (cold class is on the GPU)    */
    int32_t  coldcpu_max;
    uint64_t coldcpu_fn;
    uint64_t cold_guard_fn;      /* called before the cold pool is read, when set            */
    int32_t  cold_ffn;
    uint64_t coldffn_submit_fn;
    uint64_t coldffn_wait_fn;
} moert_cuda_config;

/* cuda.h:70 */
typedef void (*moert_cold_guard_fn)(int32_t il, const int32_t *ids, int32_t n);

/* cuda.h:80-95 (same layout) */
typedef struct moert_coldcpu_call {
    int32_t         il, kind;
    int32_t         n_cold;
    const int32_t  *cold_ids;
    const float    *x;
    int32_t         x_per_pair;
    const void     *w_host;
    uint64_t        expert_bytes;
    uint64_t        stride;
    int32_t         w_type_tag;
    int32_t         d_in, d_out;
    float          *y;
    const int32_t  *x_col;
} moert_coldcpu_call;
typedef void (*moert_coldcpu_fn)(const moert_coldcpu_call *call);

/* cuda.h:102-117 (same layout) */
typedef struct moert_coldffn_job {
    int32_t         il;
    int32_t         n_used, n_tokens;
    const int32_t  *h_counts;
    const int32_t  *h_ids;
    const int32_t  *h_cdst;
    const float    *x;
    const void     *w_gu;
    uint64_t        gu_bytes, gu_stride;
    int32_t         gu_type, d_in, d_gu;
    float          *y;
    void          (*wait_ready)(void *ev);
    void           *ev;
} moert_coldffn_job;
typedef void    (*moert_coldffn_submit_fn)(const moert_coldffn_job *job);
typedef int32_t (*moert_coldffn_wait_fn)(int32_t il, int64_t *cpu_ns);

/* cuda.h:121-131 */
static inline void moert_cuda_config_defaults(moert_cuda_config *cfg) {
    cfg->counted = 1;
    cfg->copy_stream = 0;
    cfg->coldcpu = 0;
    cfg->coldcpu_max = 3;
    cfg->coldcpu_fn = 0;
    cfg->cold_guard_fn = 0;
    cfg->cold_ffn = 0;
    cfg->coldffn_submit_fn = 0;
    cfg->coldffn_wait_fn = 0;
}

/* Copies the configuration (replaces cuda.h:135). */
void moert_cuda_configure(const moert_cuda_config *cfg);

/* cuda.h:142-146 */
enum { MOERT_MM_W_HOT = 0, MOERT_MM_W_COLD_SRC = 1, MOERT_MM_W_RAW = 2 };

/* cuda.h:150-166 (same layout). Part of the host vtable contract; this library never calls mm. */
typedef struct moert_mm_call {
    int32_t              w_sel;
    int32_t              w_type_tag;
    const void          *w_data;
    int64_t              w_n;
    const void          *b;
    int64_t              b_ncols;
    const void          *ids;
    int64_t              n_ids;
    void                *y;
    const int32_t       *ne_live;
    const void * const  *w_ptrs;
} moert_mm_call;

/* cuda.h:170-175 (same layout). pool_alloc/pool_free: device scratch, freed in strict LIFO order
 * before moert_ffn_moe returns. */
typedef struct moert_ffn_moe_host {
    void  *user;
    void *(*pool_alloc)(void *user, uint64_t nbytes);
    void  (*pool_free)(void *user, void *ptr);
    void  (*mm)(void *user, const moert_mm_call *call);
} moert_ffn_moe_host;

/* cuda.h:177-206 (same layout) */
typedef struct moert_ffn_moe_args {
    int32_t     kind;            /* 0 = merged gate_up, 1 = down                                   */
    int32_t     top_k;
    int32_t     il;
    int32_t     planc_mode;      /* only 0 (device-resident cold pool) is served                   */
    int32_t     n_used;
    int32_t     n_tokens;
    int32_t     ids_s1;          /* ids row stride in int32 elements                               */
    int32_t     d_in, d_out;
    int32_t     n_expert;
    int32_t     k;               /* hot pool slot count                                            */
    int32_t     cold_type_tag;
    uint64_t    expert_bytes;
    const void *cur;             /* f32 [d_in, 1 or n_used, n_tokens]                              */
    const void *ids;             /* i32 [n_used, n_tokens], row stride ids_s1                      */
    const void *exp_slot;        /* i32 [n_expert]                                                 */
    const void *slot_exp;        /* i32 [k]                                                        */
    const void *slot_state;      /* i32 [k]                                                        */
    const void *s_hot;           /* f32 [k] or NULL                                                */
    const void *s_cold;          /* f32 [n_expert] or NULL                                         */
    uint64_t    w_cold_dev;
    uint64_t    s_cold_dev;
    int32_t     has_w_cold;
    void       *dst;             /* f32 [d_out, n_used * n_tokens]                                 */
    void       *stream;          /* cudaStream_t                                                   */
} moert_ffn_moe_args;

/* The fused per-(layer, kind) op (replaces cuda.h:208, moert/cuda/ffn_moe.cu:892-1246).
 * The weight pools are not part of moert_ffn_moe_args in the reference (the trampoline owns the
 * ggml tensors); callers of this library bind them once per (layer, kind) with
 * moeb_bind_pools() from moeb200.h, which the trampoline does where it builds HostCtx. */
void moert_ffn_moe(const moert_ffn_moe_args *args, const moert_ffn_moe_host *host);

/* ---- host services (cuda.h:218-276); same signatures and return conventions ---- */
int32_t moert_cuda_route_counts_enable(int32_t n_layers, int32_t n_expert);
int32_t moert_cuda_route_counts_fetch(int32_t *dst, int32_t reset);
int32_t moert_cuda_host_register_pinned(void *base, uint64_t size);
void    moert_cuda_host_unregister(void *base);
int32_t moert_cuda_host_register_mapped(void *base, uint64_t size);
void   *moert_cuda_host_map(void *base, uint64_t size);

typedef struct moert_cuda_stats {
    long long fires;
    long long op_host_ns;
    long long seam_syncs;
    long long seam_ns;
    long long coldcpu_calls;
    long long coldcpu_pairs;
    long long coldcpu_ns;
    long long coldcpu_over_max;
} moert_cuda_stats;
void moert_cuda_stats_get(moert_cuda_stats *out);

int32_t moert_cuda_dir_init(int32_t sm_blocks, int32_t sm_ring_mib, int32_t sm_stage_threads);
int32_t moert_cuda_dir_async(void *dst_dev, const void *src, uint64_t nbytes);
int64_t moert_cuda_dir_mark(void);
int64_t moert_cuda_dir_poll(int32_t wait_all);
int32_t moert_cuda_publish_h2d(int32_t n, void * const *dsts, const void * const *srcs, const uint64_t *sizes);
typedef struct moert_cuda_dir_stats {
    long long async_copies, async_marks, bytes;
    long long pub_calls, pub_copies;
    long long sm_copies, sm_fallback;
    long long sm_timed, sm_gpu_ns, sm_gpu_ns_max;
    long long sm_ring_copies, sm_ring_waits; double sm_ring_wait_ms, sm_stage_ms;
} moert_cuda_dir_stats;
void    moert_cuda_dir_stats_get(moert_cuda_dir_stats *out);
int64_t moert_cuda_dir_gate(int32_t op, int64_t arg);
void    moert_cuda_set_hot_table(int32_t il, int32_t kind, const void * const *dev_ptrs, int32_t n, int32_t type_tag);

#ifdef __cplusplus
}
#endif
#endif
