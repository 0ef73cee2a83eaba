// TEST INFRASTRUCTURE — the reference's CPU sidecar (src/moe_sidecar.cpp, the survey's O2 oracle)
// driven for whole routed pair lists: one cold-FFN job per precision class (gate_up -> GeGLU ->
// down, raw down outputs, no scale and no routing weight), through moe_sidecar_ffn_submit / _wait
// (moe_sidecar.hpp:35-40). Used as a second CPU baseline for the decode configs (T <= 4: at most
// 32 pairs per job, the sidecar's PMAX). Built into oracle/_ref by `make -C oracle ref`.
#include "moe_sidecar.hpp"

#include <cstdint>
#include <cstring>

namespace {
moe_sidecar::DownPool g_down;
bool resolve_down(int32_t, moe_sidecar::DownPool *out) {
    *out = g_down;
    return g_down.base != nullptr;
}
void ready_now(void *) {}
}  // namespace

extern "C" int sidecar_init(int n_workers) { return moe_sidecar::init(n_workers) ? 1 : 0; }

// y[i][0:d_model] = down(GeGLU(gate_up(x[:, cdst[i] / n_used]))) of expert ids[i] for n pairs
// (n <= 32); the pools are [expert][rows][row bytes] host arrays of one class.
extern "C" int sidecar_ffn(int32_t il, int32_t n, const int32_t *ids, const int32_t *cdst, int32_t n_used,
                           int32_t n_tokens, const float *x, const void *w_gu, uint64_t gu_bytes, int32_t gu_type,
                           int32_t d_model, int32_t n_ff, const void *w_dn, uint64_t dn_bytes, int32_t dn_type,
                           float *y, int64_t *cpu_ns) {
    if (n <= 0 || n > 32) return 0;
    g_down = {w_dn, dn_bytes, dn_bytes, dn_type, n_ff, d_model};
    moe_sidecar::set_down_resolver(resolve_down);
    int32_t counts[2] = {0, n};
    moert_coldffn_job j = {};
    j.il = il;
    j.n_used = n_used;
    j.n_tokens = n_tokens;
    j.h_counts = counts;
    j.h_ids = ids;
    j.h_cdst = cdst;
    j.x = x;
    j.w_gu = w_gu;
    j.gu_bytes = gu_bytes;
    j.gu_stride = gu_bytes;
    j.gu_type = gu_type;
    j.d_in = d_model;
    j.d_gu = 2 * n_ff;
    j.y = y;
    j.wait_ready = ready_now;
    j.ev = nullptr;
    moe_sidecar_ffn_submit(&j);
    return moe_sidecar_ffn_wait(il, cpu_ns);
}
