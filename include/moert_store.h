/*
 * moert_store.h — the expert page store (experts.index + experts.pack), link- and file-compatible
 * with the reference's moert/include/moert/store.h:1-124 (implemented in libmoeb200.so,
 * llapis_b200/csrc/store.cpp).
 *
 * A store holds per-(layer, matrix kind, is_scale, expert) pages sliced from a source GGUF: the
 * pages the hot (Q4_K / Q5_0) class pool is filled from. The index file is a 96-byte header and
 * 72-byte records; the pack file a 32-byte header and pages starting on 256-byte boundaries, each
 * with an FNV-1a 64 checksum in its record. Little-endian hosts only, as the reference.
 *
 * Differences from the reference implementation (not from its interface or files): the reader
 * reads pages with positional reads, so one reader may serve several host threads; lookups go
 * through a hash of (layer, kind, is_scale, expert).
 */
#ifndef MOERT_STORE_H
#define MOERT_STORE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* sibling file names: "<source.gguf>" + suffix (store.h:30-31) */
#define MOERT_STORE_INDEX_SUFFIX ".experts.index"
#define MOERT_STORE_PACK_SUFFIX  ".experts.pack"

/* page record flags (store.h:34-39) */
enum moert_page_flags {
    MOERT_PAGE_REQUANTIZED = 1 << 0,  /* quant_type != source_quant */
    MOERT_PAGE_IMATRIX     = 1 << 1,
    MOERT_PAGE_PADDED      = 1 << 2,
    MOERT_PAGE_SCALE       = 1 << 3,  /* a per-expert scale page (ffn_down_exps.scale slice) */
};

/* index header facts (store.h:42-52) */
typedef struct moert_store_info {
    uint32_t format_version;
    uint64_t source_uuid;
    char     arch[16];
    int32_t  n_layers;
    int32_t  n_expert;
    uint64_t n_embd;
    uint64_t n_ff_exp;
    uint64_t pack_uuid;        /* writer: 0 = generate */
    uint64_t record_count;     /* probe only */
} moert_store_info;

/* 1 = a valid index header was read into *out, 0 = missing or invalid (store.h:55) */
int32_t moert_store_probe(const char *index_path, moert_store_info *out);
/* re-reads every page and checks its checksum: bad pages, or -1 on an I/O / format error (:60) */
int64_t moert_store_verify(const char *index_path);

/* writer (store.h:63-86): pages are appended in call order; the index is written by close */
typedef struct moert_store_writer moert_store_writer;
moert_store_writer *moert_store_writer_open(const char *index_path, const char *pack_path,
                                            const moert_store_info *info);
int32_t moert_store_writer_add_page(moert_store_writer *w, int32_t layer, int32_t expert_id, int32_t kind,
                                    int32_t is_scale, int32_t quant_type, int32_t source_quant,
                                    uint32_t extra_flags, const int64_t *shape, int32_t ndim,
                                    const void *bytes, uint64_t nbytes);
int32_t moert_store_writer_close(moert_store_writer *w);

/* FNV-1a 64 (store.h:89-91) */
uint64_t moert_store_fnv1a64(const void *data, uint64_t nbytes, uint64_t seed);
#define MOERT_STORE_FNV_SEED 14695981039346656037ull

/* reader (store.h:99-121): host-memory page reads */
typedef struct moert_store_reader moert_store_reader;
moert_store_reader *moert_store_reader_open(const char *index_path, uint64_t expect_source_uuid);
void     moert_store_reader_free(moert_store_reader *r);
int32_t  moert_store_reader_geometry(const moert_store_reader *r, int32_t *n_layers, int32_t *n_expert);
uint64_t moert_store_reader_page_nbytes(const moert_store_reader *r, int32_t layer, int32_t kind,
                                        int32_t is_scale, int32_t expert);
int32_t  moert_store_reader_page_info(const moert_store_reader *r, int32_t layer, int32_t kind,
                                      int32_t is_scale, int32_t expert, int32_t *quant_type,
                                      uint64_t *nbytes, int64_t shape[4]);
uint64_t moert_store_reader_read(moert_store_reader *r, int32_t layer, int32_t kind, int32_t is_scale,
                                 int32_t expert, void *dst, uint64_t dst_cap, int32_t verify);

#ifdef __cplusplus
}
#endif

#endif  /* MOERT_STORE_H */
