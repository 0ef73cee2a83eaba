// The expert page store: experts.index + experts.pack (include/moert_store.h), the files and the
// C ABI of the reference's moert store (moert/include/moert/store.h, moert/memmgr/store_format.h).
//
// Host-only code. The reader keeps the pack open as a file descriptor and reads pages with
// pread, so concurrent reads from several threads need no lock; records are found through a hash
// of (layer, kind, is_scale, expert).
#include "moert_store.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

// ---- on-disk layout (store_format.h:14-61): packed little-endian structs
constexpr char kIndexMagic[8] = {'E', 'X', 'I', 'D', 'X', '1', '\0', '\0'};
constexpr char kPackMagic[8] = {'E', 'X', 'P', 'A', 'C', 'K', '1', '\0'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kChecksumFnv = 1;
constexpr uint64_t kPageAlign = 256;

#pragma pack(push, 1)
struct IndexHeader {
    char magic[8];
    uint32_t format_version, header_bytes;
    uint64_t source_uuid;
    char arch[16];
    uint32_t n_layers, n_expert;
    uint64_t n_embd, n_ff_exp, pack_uuid, record_count;
    uint32_t record_stride, checksum_algo;
    uint64_t reserved;
};
struct IndexRecord {
    uint16_t layer, expert_id;
    uint8_t matrix_kind, reserved8;
    uint16_t quant_type;
    uint64_t offset, nbytes;
    int64_t shape[4];
    uint64_t checksum;
    uint16_t source_quant, reserved16;
    uint32_t flags;
};
struct PackHeader {
    char magic[8];
    uint32_t format_version, reserved32;
    uint64_t pack_uuid, reserved64;
};
#pragma pack(pop)
static_assert(sizeof(IndexHeader) == 96, "index header is 96 bytes");
static_assert(sizeof(IndexRecord) == 72, "index record is 72 bytes");
static_assert(sizeof(PackHeader) == 32, "pack header is 32 bytes");

void say(const char *fmt, const char *a, const char *b = "") { std::fprintf(stderr, fmt, a, b); }

// reads exactly n bytes at offset `off`; false on a short read or an error
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

bool header_ok(const IndexHeader &h, const char *path) {
    if (std::memcmp(h.magic, kIndexMagic, 8) != 0) return say("expert store: %s: not an experts.index file\n", path), false;
    if (h.format_version != kVersion) return say("expert store: %s: unsupported format version\n", path), false;
    if (h.header_bytes < sizeof(IndexHeader) || h.record_stride < sizeof(IndexRecord))
        return say("expert store: %s: header or record size too small\n", path), false;
    if (h.checksum_algo != kChecksumFnv) return say("expert store: %s: unknown checksum algorithm\n", path), false;
    return true;
}

// "<x>.experts.index" -> "<x>.experts.pack"; any other name -> name + ".pack"
std::string pack_path_of(const std::string &index) {
    const std::string suf = MOERT_STORE_INDEX_SUFFIX;
    if (index.size() > suf.size() && index.compare(index.size() - suf.size(), suf.size(), suf) == 0)
        return index.substr(0, index.size() - suf.size()) + MOERT_STORE_PACK_SUFFIX;
    return index + ".pack";
}

uint64_t page_key(int32_t layer, int32_t kind, int32_t is_scale, int32_t expert) {
    return ((uint64_t)(uint32_t)layer << 40) ^ ((uint64_t)(uint32_t)kind << 32) ^ ((uint64_t)(is_scale != 0) << 31) ^
           (uint64_t)(uint32_t)expert;
}

// Opens and checks an index and its pack: header, records, the pack header and the uuid link.
struct Store {
    IndexHeader hdr{};
    std::vector<IndexRecord> recs;
    int pack_fd = -1;
    uint64_t pack_bytes = 0;
    // whether record r's page lies inside the pack (offset + nbytes without overflow)
    bool in_pack(const IndexRecord &r) const {
        uint64_t end = 0;
        return !__builtin_add_overflow(r.offset, r.nbytes, &end) && end <= pack_bytes;
    }
};

bool load_store(const char *index_path, Store &s) {
    FILE *f = std::fopen(index_path, "rb");
    if (!f) return say("expert store: cannot open %s\n", index_path), false;
    bool ok = std::fread(&s.hdr, 1, sizeof(s.hdr), f) == sizeof(s.hdr);
    if (!ok) say("expert store: %s: truncated header\n", index_path);
    ok = ok && header_ok(s.hdr, index_path);
    if (ok) {
        // the record list must fit in the file before anything is sized from the header's count
        std::fseek(f, 0, SEEK_END);
        const long fsz = std::ftell(f);
        uint64_t need = 0;
        if (fsz < 0 || __builtin_mul_overflow(s.hdr.record_count, (uint64_t)s.hdr.record_stride, &need) ||
            __builtin_add_overflow(need, (uint64_t)s.hdr.header_bytes, &need) || need > (uint64_t)fsz) {
            say("expert store: %s: record list longer than the file\n", index_path);
            ok = false;
        }
    }
    if (ok && std::fseek(f, (long)s.hdr.header_bytes, SEEK_SET) != 0) ok = false;
    if (ok) {
        s.recs.resize(s.hdr.record_count);
        std::vector<uint8_t> rec(s.hdr.record_stride);
        for (uint64_t i = 0; ok && i < s.hdr.record_count; ++i) {
            if (std::fread(rec.data(), 1, rec.size(), f) != rec.size()) {
                say("expert store: %s: truncated record list\n", index_path);
                ok = false;
            } else {
                std::memcpy(&s.recs[i], rec.data(), sizeof(IndexRecord));   // unknown record tails skipped
            }
        }
    }
    std::fclose(f);
    if (!ok) return false;
    const std::string pp = pack_path_of(index_path);
    s.pack_fd = ::open(pp.c_str(), O_RDONLY | O_CLOEXEC);
    if (s.pack_fd < 0) return say("expert store: cannot open pack %s\n", pp.c_str()), false;
    struct stat st{};
    s.pack_bytes = ::fstat(s.pack_fd, &st) == 0 ? (uint64_t)st.st_size : 0;
    PackHeader ph{};
    if (!pread_all(s.pack_fd, &ph, sizeof(ph), 0) || std::memcmp(ph.magic, kPackMagic, 8) != 0 ||
        ph.format_version != kVersion) {
        say("expert store: %s: bad pack header\n", pp.c_str());
    } else if (ph.pack_uuid != s.hdr.pack_uuid) {
        say("expert store: %s does not belong to %s (pack uuid differs)\n", pp.c_str(), index_path);
    } else {
        return true;
    }
    ::close(s.pack_fd);
    s.pack_fd = -1;
    return false;
}

}  // namespace

struct moert_store_reader {
    Store s;
    std::unordered_map<uint64_t, uint32_t> at;   // page key -> record
};

struct moert_store_writer {
    std::string index_path;
    FILE *pack = nullptr;
    IndexHeader hdr{};
    std::vector<IndexRecord> recs;
    uint64_t pos = 0;       // bytes written to the pack so far
    bool failed = false;
};

extern "C" uint64_t moert_store_fnv1a64(const void *data, uint64_t nbytes, uint64_t seed) {
    // FNV-1a, 64-bit: xor the byte in, then multiply by the FNV prime 2^40 + 2^8 + 0xb3
    const uint8_t *p = static_cast<const uint8_t *>(data);
    uint64_t h = seed;
    for (uint64_t i = 0; i < nbytes; ++i) h = (h ^ p[i]) * 0x100000001b3ull;
    return h;
}

extern "C" int32_t moert_store_probe(const char *index_path, moert_store_info *out) {
    if (!index_path || !out) return 0;
    FILE *f = std::fopen(index_path, "rb");
    if (!f) return 0;   // quiet: used to look for a sibling store
    IndexHeader h{};
    const bool ok = std::fread(&h, 1, sizeof(h), f) == sizeof(h) && header_ok(h, index_path);
    std::fclose(f);
    if (!ok) return 0;
    out->format_version = h.format_version;
    out->source_uuid = h.source_uuid;
    std::memcpy(out->arch, h.arch, sizeof(out->arch));
    out->arch[sizeof(out->arch) - 1] = '\0';
    out->n_layers = (int32_t)h.n_layers;
    out->n_expert = (int32_t)h.n_expert;
    out->n_embd = h.n_embd;
    out->n_ff_exp = h.n_ff_exp;
    out->pack_uuid = h.pack_uuid;
    out->record_count = h.record_count;
    return 1;
}

extern "C" int64_t moert_store_verify(const char *index_path) {
    if (!index_path) return -1;
    Store s;
    if (!load_store(index_path, s)) return -1;
    std::vector<uint8_t> buf;
    int64_t bad = 0;
    for (size_t i = 0; i < s.recs.size(); ++i) {
        const IndexRecord &r = s.recs[i];
        const bool inside = s.in_pack(r);
        if (inside) buf.resize(r.nbytes);
        const bool read = inside && pread_all(s.pack_fd, buf.data(), r.nbytes, r.offset);
        if (!read || moert_store_fnv1a64(buf.data(), r.nbytes, MOERT_STORE_FNV_SEED) != r.checksum) {
            std::fprintf(stderr, "expert store: page %zu (layer %u, expert %u, kind %u%s): %s\n", i, r.layer, r.expert_id,
                         r.matrix_kind, (r.flags & MOERT_PAGE_SCALE) ? ", scale" : "",
                         read ? "checksum mismatch" : "read failed");
            ++bad;
        }
    }
    ::close(s.pack_fd);
    return bad;
}

extern "C" moert_store_reader *moert_store_reader_open(const char *index_path, uint64_t expect_source_uuid) {
    if (!index_path) return nullptr;
    auto *r = new moert_store_reader();
    if (!load_store(index_path, r->s)) {
        delete r;
        return nullptr;
    }
    if (expect_source_uuid && r->s.hdr.source_uuid != expect_source_uuid) {
        std::fprintf(stderr, "expert store: %s was sliced from another source (uuid %016" PRIx64 ", want %016" PRIx64 ")\n",
                     index_path, r->s.hdr.source_uuid, expect_source_uuid);
        ::close(r->s.pack_fd);
        delete r;
        return nullptr;
    }
    const IndexHeader &h = r->s.hdr;
    for (uint32_t i = 0; i < r->s.recs.size(); ++i) {
        const IndexRecord &rec = r->s.recs[i];
        // the reference's reader addresses kinds 0..3 of in-range layers and experts; a later record
        // for the same page replaces an earlier one
        if (rec.layer >= h.n_layers || rec.expert_id >= h.n_expert || rec.matrix_kind >= 4) continue;
        r->at[page_key(rec.layer, rec.matrix_kind, (rec.flags & MOERT_PAGE_SCALE) ? 1 : 0, rec.expert_id)] = i;
    }
    return r;
}

extern "C" void moert_store_reader_free(moert_store_reader *r) {
    if (!r) return;
    if (r->s.pack_fd >= 0) ::close(r->s.pack_fd);
    delete r;
}

extern "C" int32_t moert_store_reader_geometry(const moert_store_reader *r, int32_t *n_layers, int32_t *n_expert) {
    if (!r) return 0;
    if (n_layers) *n_layers = (int32_t)r->s.hdr.n_layers;
    if (n_expert) *n_expert = (int32_t)r->s.hdr.n_expert;
    return 1;
}

static const IndexRecord *find_page(const moert_store_reader *r, int32_t layer, int32_t kind, int32_t is_scale,
                                    int32_t expert) {
    if (!r || is_scale < 0 || is_scale > 1) return nullptr;
    const auto it = r->at.find(page_key(layer, kind, is_scale, expert));
    return it == r->at.end() ? nullptr : &r->s.recs[it->second];
}

extern "C" uint64_t moert_store_reader_page_nbytes(const moert_store_reader *r, int32_t layer, int32_t kind,
                                                   int32_t is_scale, int32_t expert) {
    const IndexRecord *rec = find_page(r, layer, kind, is_scale, expert);
    return rec ? rec->nbytes : 0;
}

extern "C" int32_t moert_store_reader_page_info(const moert_store_reader *r, int32_t layer, int32_t kind,
                                                int32_t is_scale, int32_t expert, int32_t *quant_type,
                                                uint64_t *nbytes, int64_t shape[4]) {
    const IndexRecord *rec = find_page(r, layer, kind, is_scale, expert);
    if (!rec) return 0;
    if (quant_type) *quant_type = (int32_t)rec->quant_type;
    if (nbytes) *nbytes = rec->nbytes;
    if (shape) std::memcpy(shape, rec->shape, sizeof(rec->shape));
    return 1;
}

extern "C" uint64_t moert_store_reader_read(moert_store_reader *r, int32_t layer, int32_t kind, int32_t is_scale,
                                            int32_t expert, void *dst, uint64_t dst_cap, int32_t verify) {
    if (!dst) return 0;
    const IndexRecord *rec = find_page(r, layer, kind, is_scale, expert);
    if (!rec) return 0;
    if (rec->nbytes > dst_cap) {
        std::fprintf(stderr, "expert store: page of %" PRIu64 " bytes does not fit %" PRIu64 " (layer %d, expert %d)\n",
                     rec->nbytes, dst_cap, layer, expert);
        return 0;
    }
    if (!r->s.in_pack(*rec) || !pread_all(r->s.pack_fd, dst, rec->nbytes, rec->offset)) {
        std::fprintf(stderr, "expert store: page read failed (layer %d, expert %d, kind %d)\n", layer, expert, kind);
        return 0;
    }
    if (verify && moert_store_fnv1a64(dst, rec->nbytes, MOERT_STORE_FNV_SEED) != rec->checksum) {
        std::fprintf(stderr, "expert store: checksum mismatch (layer %d, expert %d, kind %d)\n", layer, expert, kind);
        return 0;
    }
    return rec->nbytes;
}

extern "C" moert_store_writer *moert_store_writer_open(const char *index_path, const char *pack_path,
                                                       const moert_store_info *info) {
    if (!index_path || !pack_path || !info || info->n_layers <= 0 || info->n_expert <= 0) return nullptr;
    auto *w = new moert_store_writer();
    w->index_path = index_path;
    w->pack = std::fopen(pack_path, "wb");
    if (!w->pack) {
        say("expert store: cannot create %s\n", pack_path);
        delete w;
        return nullptr;
    }
    IndexHeader &h = w->hdr;
    std::memcpy(h.magic, kIndexMagic, 8);
    h.format_version = kVersion;
    h.header_bytes = sizeof(IndexHeader);
    h.source_uuid = info->source_uuid;
    std::strncpy(h.arch, info->arch, sizeof(h.arch) - 1);
    h.n_layers = (uint32_t)info->n_layers;
    h.n_expert = (uint32_t)info->n_expert;
    h.n_embd = info->n_embd;
    h.n_ff_exp = info->n_ff_exp;
    // a generated uuid: the index path hashed with the clock, so stores written to the same path
    // at different times do not pair with each other's packs
    const uint64_t now = (uint64_t)std::chrono::system_clock::now().time_since_epoch().count();
    h.pack_uuid = info->pack_uuid ? info->pack_uuid
                                  : moert_store_fnv1a64(index_path, std::strlen(index_path), MOERT_STORE_FNV_SEED ^ now);
    h.record_stride = sizeof(IndexRecord);
    h.checksum_algo = kChecksumFnv;
    PackHeader ph{};
    std::memcpy(ph.magic, kPackMagic, 8);
    ph.format_version = kVersion;
    ph.pack_uuid = h.pack_uuid;
    if (std::fwrite(&ph, 1, sizeof(ph), w->pack) != sizeof(ph)) {
        say("expert store: cannot write %s\n", pack_path);
        std::fclose(w->pack);
        delete w;
        return nullptr;
    }
    w->pos = sizeof(ph);
    return w;
}

extern "C" int32_t moert_store_writer_add_page(moert_store_writer *w, int32_t layer, int32_t expert_id, int32_t kind,
                                               int32_t is_scale, int32_t quant_type, int32_t source_quant,
                                               uint32_t extra_flags, const int64_t *shape, int32_t ndim,
                                               const void *bytes, uint64_t nbytes) {
    if (!w) return 0;
    const bool args_ok = !w->failed && bytes && nbytes > 0 && shape && ndim >= 1 && ndim <= 4 && layer >= 0 &&
                         layer < (int32_t)w->hdr.n_layers && expert_id >= 0 && expert_id < (int32_t)w->hdr.n_expert &&
                         kind >= 0 && kind <= 255;
    if (!args_ok) {
        w->failed = true;   // a failed writer produces no index
        return 0;
    }
    const uint64_t at = (w->pos + kPageAlign - 1) / kPageAlign * kPageAlign;
    static const uint8_t zero[kPageAlign] = {};
    if ((at > w->pos && std::fwrite(zero, 1, at - w->pos, w->pack) != at - w->pos) ||
        std::fwrite(bytes, 1, nbytes, w->pack) != nbytes) {
        w->failed = true;
        return 0;
    }
    w->pos = at + nbytes;
    IndexRecord r{};
    r.layer = (uint16_t)layer;
    r.expert_id = (uint16_t)expert_id;
    r.matrix_kind = (uint8_t)kind;
    r.quant_type = (uint16_t)quant_type;
    r.offset = at;
    r.nbytes = nbytes;
    for (int i = 0; i < 4; ++i) r.shape[i] = i < ndim ? shape[i] : 1;
    r.checksum = moert_store_fnv1a64(bytes, nbytes, MOERT_STORE_FNV_SEED);
    r.source_quant = (uint16_t)source_quant;
    r.flags = extra_flags | (is_scale ? (uint32_t)MOERT_PAGE_SCALE : 0u) |
              (quant_type != source_quant ? (uint32_t)MOERT_PAGE_REQUANTIZED : 0u);
    w->recs.push_back(r);
    return 1;
}

extern "C" int32_t moert_store_writer_close(moert_store_writer *w) {
    if (!w) return 0;
    bool ok = !w->failed;
    if (std::fflush(w->pack) != 0 || std::ferror(w->pack)) ok = false;
    if (std::fclose(w->pack) != 0) ok = false;
    if (ok) {
        w->hdr.record_count = w->recs.size();
        FILE *f = std::fopen(w->index_path.c_str(), "wb");
        ok = f != nullptr;
        if (f) {
            ok = std::fwrite(&w->hdr, 1, sizeof(w->hdr), f) == sizeof(w->hdr) &&
                 (w->recs.empty() || std::fwrite(w->recs.data(), sizeof(IndexRecord), w->recs.size(), f) == w->recs.size());
            if (std::fflush(f) != 0 || std::ferror(f)) ok = false;
            if (std::fclose(f) != 0) ok = false;
        }
    }
    if (!ok) say("expert store: writing %s failed; the store is not usable\n", w->index_path.c_str());
    delete w;
    return ok ? 1 : 0;
}
