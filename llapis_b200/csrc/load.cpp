// Expert loading from files into the HBM class pools (include/moeb200.h, "Expert loading"):
//  - a GGUF tensor directory (the reference's format: third_party/llama/ggml/src/gguf.cpp, v2/v3):
//    header, key/values, tensor infos, the data section at the next `general.alignment` boundary;
//    a Gemma-4 layer's stacked expert tensors are [E][rows][row bytes], the pool layout itself;
//  - file byte ranges and expert-store pages copied to device memory by eight reader threads, each
//    with two pinned staging buffers and its own copy stream, so reads run in parallel and each
//    overlaps the host-to-device copies in flight.
// Host code; the device is reached only through cudaMemcpyAsync on the workers' streams, which
// start after the caller's stream's earlier work and have all completed when a loader returns.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "moeb200.h"
#include "moert_store.h"
#include "params.h"

using moeb::set_last_error;

namespace {

// ggml type id -> (values per block, bytes per block) (the type traits of ggml.c); 0 = unknown
struct TypeSize {
    int32_t blck, bytes;
};
TypeSize type_size(int32_t t) {
    switch (t) {
        case 0: return {1, 4};        // F32
        case 1: return {1, 2};        // F16
        case 2: return {32, 18};      // Q4_0
        case 3: return {32, 20};      // Q4_1
        case 6: return {32, 22};      // Q5_0
        case 7: return {32, 24};      // Q5_1
        case 8: return {32, 34};      // Q8_0
        case 9: return {32, 36};      // Q8_1
        case 10: return {256, 84};    // Q2_K
        case 11: return {256, 110};   // Q3_K
        case 12: return {256, 144};   // Q4_K
        case 13: return {256, 176};   // Q5_K
        case 14: return {256, 210};   // Q6_K
        case 15: return {256, 292};   // Q8_K
        case 16: return {256, 66};    // IQ2_XXS
        case 17: return {256, 74};    // IQ2_XS
        case 18: return {256, 98};    // IQ3_XXS
        case 19: return {256, 50};    // IQ1_S
        case 20: return {32, 18};     // IQ4_NL
        case 21: return {256, 110};   // IQ3_S
        case 22: return {256, 82};    // IQ2_S
        case 23: return {256, 136};   // IQ4_XS
        case 24: return {1, 1};       // I8
        case 25: return {1, 2};       // I16
        case 26: return {1, 4};       // I32
        case 27: return {1, 8};       // I64
        case 28: return {1, 8};       // F64
        case 29: return {256, 56};    // IQ1_M
        case 30: return {1, 2};       // BF16
        default: return {0, 0};
    }
}

// buffered little-endian reader over a FILE of `size` bytes; every length read from the file is
// checked against the bytes left before it is used, so a corrupt header ends the parse instead of
// seeking backwards or allocating what the file cannot hold
struct In {
    FILE *f;
    uint64_t size = 0;
    uint64_t pos = 0;
    bool ok = true;
    uint64_t left() const { return pos <= size ? size - pos : 0; }
    template <class T> T get() {
        T v{};
        if (ok && std::fread(&v, sizeof(T), 1, f) == 1) pos += sizeof(T);
        else ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 24) || n > left()) return ok = false, std::string();
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        pos += n;
        return s;
    }
    void skip(uint64_t n) {
        if (ok && n <= left() && std::fseek(f, (long)n, SEEK_CUR) == 0) pos += n;
        else ok = false;
    }
};

enum { kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kStr, kArr, kU64, kI64, kF64 };
int scalar_bytes(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

struct Kv {
    uint32_t type = 0;
    uint64_t u = 0;      // integer value (sign-extended for signed types)
    double f = 0.0;      // float value
    std::string s;       // string value
};

}  // namespace

struct moeb_gguf {
    std::string path;
    uint32_t alignment = 32;
    uint64_t data_offset = 0;
    std::unordered_map<std::string, Kv> kv;
    std::unordered_map<std::string, moeb_gguf_tensor> tensors;
};

extern "C" moeb_gguf *moeb_gguf_open(const char *path) {
    if (!path) return set_last_error(MOEB_EINVAL, "moeb_gguf_open: null path"), nullptr;
    FILE *f = std::fopen(path, "rb");
    if (!f) return set_last_error(MOEB_EINVAL, "moeb_gguf_open: cannot open %s", path), nullptr;
    std::fseek(f, 0, SEEK_END);
    const long fsize = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    In in{f, fsize > 0 ? (uint64_t)fsize : 0};
    auto *g = new moeb_gguf();
    g->path = path;
    const uint32_t magic = in.get<uint32_t>(), version = in.get<uint32_t>();
    const uint64_t n_tensors = in.get<uint64_t>(), n_kv = in.get<uint64_t>();
    const char *err = nullptr;
    if (!in.ok || std::memcmp(&magic, "GGUF", 4) != 0) err = "not a GGUF file";
    else if (version < 2 || version > 3) err = "unsupported GGUF version";
    for (uint64_t i = 0; !err && i < n_kv; ++i) {
        const std::string key = in.str();
        Kv v;
        v.type = in.get<uint32_t>();
        if (v.type == kStr) {
            v.s = in.str();
        } else if (v.type == kArr) {   // arrays are skipped (the loader needs none)
            const uint32_t et = in.get<uint32_t>();
            const uint64_t n = in.get<uint64_t>();
            if (et == kStr) {
                if (n > in.left() / 8) err = "array longer than the file";   // every string has an 8-byte length
                for (uint64_t j = 0; !err && j < n && in.ok; ++j) in.str();
            } else if (scalar_bytes(et)) {
                if (n > in.left() / (uint64_t)scalar_bytes(et)) err = "array longer than the file";
                else in.skip(n * (uint64_t)scalar_bytes(et));
            } else {
                err = "bad array element type";
            }
        } else if (const int nb = scalar_bytes(v.type)) {
            uint64_t raw = 0;
            for (int b = 0; b < nb; ++b) raw |= (uint64_t)in.get<uint8_t>() << (8 * b);
            switch (v.type) {
                case kI8: v.u = (uint64_t)(int64_t)(int8_t)raw; break;
                case kI16: v.u = (uint64_t)(int64_t)(int16_t)raw; break;
                case kI32: v.u = (uint64_t)(int64_t)(int32_t)raw; break;
                default: v.u = raw;
            }
            if (v.type == kF32) { float x; uint32_t r32 = (uint32_t)raw; std::memcpy(&x, &r32, 4); v.f = x; }
            if (v.type == kF64) std::memcpy(&v.f, &raw, 8);
        } else {
            err = "bad key/value type";
        }
        if (!in.ok) err = "truncated key/values";
        if (!err) g->kv[key] = v;
    }
    if (!err) {
        const auto it = g->kv.find("general.alignment");
        if (it != g->kv.end()) g->alignment = (uint32_t)it->second.u;
        if (g->alignment == 0 || (g->alignment & (g->alignment - 1)) != 0) err = "alignment is not a power of two";
    }
    std::vector<std::pair<std::string, moeb_gguf_tensor>> infos;
    for (uint64_t i = 0; !err && i < n_tensors; ++i) {
        moeb_gguf_tensor t{};
        const std::string name = in.str();
        t.n_dims = (int32_t)in.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) { err = "tensor with more than 4 dimensions"; break; }
        for (int d = 0; d < 4; ++d) t.ne[d] = d < t.n_dims ? in.get<int64_t>() : 1;
        t.type = (int32_t)in.get<uint32_t>();
        t.offset = in.get<uint64_t>();
        if (!in.ok) { err = "truncated tensor infos"; break; }
        const TypeSize ts = type_size(t.type);
        if (ts.blck == 0 || t.ne[0] % ts.blck != 0 || t.ne[0] < 0 || t.ne[1] < 0 || t.ne[2] < 0 || t.ne[3] < 0) {
            err = "tensor of an unknown type or a row that is not whole blocks";
            break;
        }
        uint64_t nb = (uint64_t)(t.ne[0] / ts.blck);
        bool ovf = __builtin_mul_overflow(nb, (uint64_t)ts.bytes, &nb);
        for (int d = 1; d < 4; ++d) ovf = ovf || __builtin_mul_overflow(nb, (uint64_t)t.ne[d], &nb);
        if (ovf) { err = "tensor size overflows"; break; }
        t.nbytes = nb;
        infos.emplace_back(name, t);
    }
    if (!err) {
        g->data_offset = n_tensors ? (in.pos + g->alignment - 1) / g->alignment * g->alignment : in.pos;
        const uint64_t size = in.size;
        for (auto &nt : infos) {
            uint64_t end = 0;
            if (__builtin_add_overflow(nt.second.offset, g->data_offset, &nt.second.offset) ||   // absolute
                __builtin_add_overflow(nt.second.offset, nt.second.nbytes, &end) || end > size) {
                err = "tensor data past the end of the file";
                break;
            }
            g->tensors[nt.first] = nt.second;
        }
    }
    std::fclose(f);
    if (err) {
        set_last_error(MOEB_EINVAL, "moeb_gguf_open: %s: %s", path, err);
        delete g;
        return nullptr;
    }
    return g;
}

extern "C" void moeb_gguf_close(moeb_gguf *g) { delete g; }

extern "C" int moeb_gguf_find_tensor(const moeb_gguf *g, const char *name, moeb_gguf_tensor *out) {
    if (!g || !name || !out) return set_last_error(MOEB_EINVAL, "moeb_gguf_find_tensor: null argument");
    const auto it = g->tensors.find(name);
    if (it == g->tensors.end()) return set_last_error(MOEB_EINVAL, "tensor %s not in %s", name, g->path.c_str());
    *out = it->second;
    return MOEB_OK;
}

static const Kv *find_kv(const moeb_gguf *g, const char *key) {
    if (!g || !key) return nullptr;
    const auto it = g->kv.find(key);
    return it == g->kv.end() ? nullptr : &it->second;
}

extern "C" int moeb_gguf_get_u32(const moeb_gguf *g, const char *key, uint32_t *out) {
    const Kv *v = find_kv(g, key);
    if (!v || !out) return set_last_error(MOEB_EINVAL, "key %s not found", key ? key : "(null)");
    if (v->type == kStr || v->type == kArr || v->type == kF32 || v->type == kF64 || v->u > 0xffffffffull)
        return set_last_error(MOEB_EINVAL, "key %s is not an unsigned 32-bit integer", key);
    *out = (uint32_t)v->u;
    return MOEB_OK;
}

extern "C" int moeb_gguf_get_f32(const moeb_gguf *g, const char *key, float *out) {
    const Kv *v = find_kv(g, key);
    if (!v || !out) return set_last_error(MOEB_EINVAL, "key %s not found", key ? key : "(null)");
    if (v->type != kF32 && v->type != kF64) return set_last_error(MOEB_EINVAL, "key %s is not a float", key);
    *out = (float)v->f;
    return MOEB_OK;
}

extern "C" int moeb_gguf_get_str(const moeb_gguf *g, const char *key, char *out, size_t cap) {
    const Kv *v = find_kv(g, key);
    if (!v || !out || cap == 0) return set_last_error(MOEB_EINVAL, "key %s not found", key ? key : "(null)");
    if (v->type != kStr) return set_last_error(MOEB_EINVAL, "key %s is not a string", key);
    if (v->s.size() + 1 > cap) return set_last_error(MOEB_ESPACE, "key %s: value longer than %zu bytes", key, cap - 1);
    std::memcpy(out, v->s.c_str(), v->s.size() + 1);
    return MOEB_OK;
}

// ---------------------------------------------------------------- host -> device through pinned staging
namespace {

constexpr uint64_t kChunk = 8u << 20;   // bytes per staging buffer
constexpr int kWorkers = 8;             // reader threads, two staging buffers each

// The pinned staging buffers: allocated on first use (portable, so any device may copy from them)
// and kept for the process; one staged copy runs at a time.
struct Staging {
    std::mutex mu;
    void *buf[kWorkers][2] = {};
    bool ready = false;
};
Staging g_stage;

// Copies `n` pieces to the device: piece i is produced into pinned memory by fill(i, buf, cap)
// (returning its length, 0 on failure; called from several threads at once) and copied to dst(i).
// Worker w takes pieces w, w + W, ... on its own stream, alternating its two buffers; a buffer is
// refilled once the copy out of it has completed. Every copy has completed on return.
template <class Fill, class Dst>
int64_t staged_copy(int n, uint64_t cap, Fill fill, Dst dst, cudaStream_t s) {
    if (cap > kChunk) return set_last_error(MOEB_EINVAL, "expert load: piece of %llu bytes exceeds the %llu-byte staging",
                                            (unsigned long long)cap, (unsigned long long)kChunk);
    std::lock_guard<std::mutex> lk(g_stage.mu);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    for (int w = 0; e == cudaSuccess && !g_stage.ready && w < kWorkers; ++w)
        for (int b = 0; e == cudaSuccess && b < 2; ++b)
            if (!g_stage.buf[w][b]) e = cudaHostAlloc(&g_stage.buf[w][b], kChunk, cudaHostAllocPortable);
    if (e != cudaSuccess) return set_last_error(MOEB_ECUDA, "expert load staging: %s", cudaGetErrorString(e));
    g_stage.ready = true;
    const int W = n < kWorkers ? n : kWorkers;
    cudaStream_t ws[kWorkers] = {};
    cudaEvent_t ev[kWorkers][2] = {}, start = nullptr;
    e = cudaEventCreateWithFlags(&start, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(start, s);   // after the caller's earlier work on `s`
    for (int w = 0; e == cudaSuccess && w < W; ++w) {
        e = cudaStreamCreateWithFlags(&ws[w], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ws[w], start, 0);
        for (int b = 0; e == cudaSuccess && b < 2; ++b) e = cudaEventCreateWithFlags(&ev[w][b], cudaEventDisableTiming);
    }
    std::atomic<int64_t> total{0};
    std::atomic<int> bad_piece{-1};
    std::atomic<int> cuda_err{(int)e};
    if (e == cudaSuccess) {
        std::vector<std::thread> th;
        for (int w = 0; w < W; ++w)
            th.emplace_back([&, w]() {
                cudaError_t we = cudaSetDevice(dev);
                for (int i = w, k = 0; we == cudaSuccess && i < n; i += W, ++k) {
                    if (bad_piece.load() >= 0 || cuda_err.load() != cudaSuccess) break;
                    const int b = k & 1;
                    if (k >= 2 && (we = cudaEventSynchronize(ev[w][b])) != cudaSuccess) break;
                    const uint64_t got = fill(i, g_stage.buf[w][b], cap);
                    if (got == 0) {
                        bad_piece.store(i);
                        break;
                    }
                    we = cudaMemcpyAsync(dst(i), g_stage.buf[w][b], got, cudaMemcpyHostToDevice, ws[w]);
                    if (we == cudaSuccess) we = cudaEventRecord(ev[w][b], ws[w]);
                    total += (int64_t)got;
                }
                if (we != cudaSuccess) cuda_err.store((int)we);
            });
        for (auto &t : th) t.join();
    }
    for (int w = 0; w < W; ++w) {   // the staging buffers are reused by the next call
        if (ws[w]) {
            const cudaError_t e2 = cudaStreamSynchronize(ws[w]);
            if (e2 != cudaSuccess) cuda_err.store((int)e2);
            cudaStreamDestroy(ws[w]);
        }
        for (int b = 0; b < 2; ++b)
            if (ev[w][b]) cudaEventDestroy(ev[w][b]);
    }
    if (start) cudaEventDestroy(start);
    if (cuda_err.load() != cudaSuccess)
        return set_last_error(MOEB_ECUDA, "expert load: %s", cudaGetErrorString((cudaError_t)cuda_err.load()));
    if (bad_piece.load() >= 0) return set_last_error(MOEB_EINVAL, "expert load: read of piece %d failed", bad_piece.load());
    return total.load();
}

bool pread_all(int fd, void *dst, uint64_t n, uint64_t off) {
    uint8_t *p = static_cast<uint8_t *>(dst);
    while (n > 0) {
        const ssize_t got = ::pread(fd, p, n, (off_t)off);
        if (got <= 0) return false;
        p += got;
        n -= (uint64_t)got;
        off += (uint64_t)got;
    }
    return true;
}

}  // namespace

extern "C" int64_t moeb_load_file_range(const char *path, uint64_t offset, uint64_t nbytes, void *dst, void *stream) {
    if (!path || !dst) return set_last_error(MOEB_EINVAL, "moeb_load_file_range: null path or destination");
    if (nbytes == 0) return 0;
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_last_error(MOEB_EINVAL, "moeb_load_file_range: cannot open %s", path);
    const int n = (int)((nbytes + kChunk - 1) / kChunk);
    const int64_t r = staged_copy(
        n, kChunk,
        [&](int i, void *buf, uint64_t) -> uint64_t {
            const uint64_t at = (uint64_t)i * kChunk, len = nbytes - at < kChunk ? nbytes - at : kChunk;
            return pread_all(fd, buf, len, offset + at) ? len : 0;
        },
        [&](int i) { return static_cast<uint8_t *>(dst) + (uint64_t)i * kChunk; }, (cudaStream_t)stream);
    ::close(fd);
    return r;
}

extern "C" int64_t moeb_load_store_pages(struct moert_store_reader *r, int32_t layer, int32_t kind, int32_t is_scale,
                                         const int32_t *experts, int32_t n, void *dst, uint64_t dst_stride,
                                         int32_t verify, void *stream) {
    if (!r || !experts || !dst || n < 0) return set_last_error(MOEB_EINVAL, "moeb_load_store_pages: null argument");
    uint64_t cap = 0;
    for (int i = 0; i < n; ++i) {
        const uint64_t nb = moert_store_reader_page_nbytes(r, layer, kind, is_scale, experts[i]);
        if (nb == 0)
            return set_last_error(MOEB_EINVAL, "store has no page for layer %d, kind %d%s, expert %d", layer, kind,
                                  is_scale ? " (scale)" : "", experts[i]);
        if (nb > dst_stride)
            return set_last_error(MOEB_EINVAL, "page of %llu bytes exceeds the slot stride %llu", (unsigned long long)nb,
                                  (unsigned long long)dst_stride);
        cap = nb > cap ? nb : cap;
    }
    if (n == 0) return 0;
    return staged_copy(
        n, cap,
        [&](int i, void *buf, uint64_t c) -> uint64_t {
            return moert_store_reader_read(r, layer, kind, is_scale, experts[i], buf, c, verify);
        },
        [&](int i) { return static_cast<uint8_t *>(dst) + (uint64_t)i * dst_stride; }, (cudaStream_t)stream);
}
