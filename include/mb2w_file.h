/* Reader for MB2W weight files (cpu_mamba_b200.export.save): the flat export
 * format of a Mamba block or residual stack -- the "ggml/ONNX-style export"
 * on the reference's roadmap (README.md:203).  Header only, C99, no
 * allocation: map or read the file, call mb2w_parse, then point an mb2_block
 * descriptor's fields at device copies of the tensors it finds.
 *
 * Layout (little endian, offsets from the start of the file): a 32-byte
 * header, n_meta 48-byte (key, value) records, n_tensors 144-byte tensor
 * records, then each tensor's bytes at a 64-byte aligned offset. */
#ifndef MB2W_FILE_H
#define MB2W_FILE_H

#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define MB2W_VERSION 1

typedef struct {
    char magic[4]; /* "MB2W" */
    uint32_t version, n_meta, n_tensors;
    uint64_t data_offset, file_bytes;
} mb2w_header;

typedef struct {
    char key[40]; /* NUL padded: kind, n_layers, d_model, d_inner, d_state,
                     d_conv, dt_rank, conv_bias, bias, eps_1e12, dtype */
    int64_t value;
} mb2w_meta;

enum { MB2W_F32 = 0, MB2W_BF16 = 1, MB2W_I8 = 2, MB2W_U8 = 3, MB2W_F16 = 4 };

typedef struct {
    char name[64];      /* state_dict key, e.g. "layers.3.mixer.in_proj.weight_q" */
    uint32_t dtype;     /* MB2W_* */
    uint32_t ndim;
    int64_t shape[4];
    uint64_t offset;    /* from the start of the file, 64-byte aligned */
    uint64_t nbytes;
    int32_t scheme;     /* 0 dense, 1 int8, 2 int4, 3 nf4 (MB2_Q_* of mamba_b200.h) */
    int32_t group_size; /* 0: one scale per row */
    int64_t in_dim;     /* unpacked input width of a quantised weight */
    uint8_t reserved[8];
} mb2w_tensor;

typedef char mb2w_header_is_32_bytes[sizeof(mb2w_header) == 32 ? 1 : -1];
typedef char mb2w_meta_is_48_bytes[sizeof(mb2w_meta) == 48 ? 1 : -1];
typedef char mb2w_tensor_is_144_bytes[sizeof(mb2w_tensor) == 144 ? 1 : -1];

/* 0 on success; -1 not an MB2W file or unknown version, -2 truncated, -3 a
 * tensor outside the file. */
static inline int mb2w_parse(const void *file, size_t size, const mb2w_header **hdr,
                             const mb2w_meta **meta, const mb2w_tensor **tensors) {
    const char *base = (const char *)file;
    const mb2w_header *h = (const mb2w_header *)base;
    if (size < sizeof(mb2w_header) || memcmp(h->magic, "MB2W", 4) != 0 ||
        h->version != MB2W_VERSION)
        return -1;
    const size_t table = sizeof(mb2w_header) + (size_t)h->n_meta * sizeof(mb2w_meta) +
                         (size_t)h->n_tensors * sizeof(mb2w_tensor);
    if (size < h->file_bytes || size < table) return -2;
    const mb2w_tensor *t = (const mb2w_tensor *)(base + sizeof(mb2w_header) +
                                                 (size_t)h->n_meta * sizeof(mb2w_meta));
    for (uint32_t i = 0; i < h->n_tensors; ++i)
        if (t[i].offset + t[i].nbytes > h->file_bytes) return -3;
    *hdr = h;
    *meta = (const mb2w_meta *)(base + sizeof(mb2w_header));
    *tensors = t;
    return 0;
}

static inline int64_t mb2w_meta_get(const mb2w_header *h, const mb2w_meta *meta,
                                    const char *key, int64_t fallback) {
    for (uint32_t i = 0; i < h->n_meta; ++i)
        if (strncmp(meta[i].key, key, sizeof(meta[i].key)) == 0) return meta[i].value;
    return fallback;
}

static inline const mb2w_tensor *mb2w_find(const mb2w_header *h, const mb2w_tensor *tensors,
                                           const char *name) {
    for (uint32_t i = 0; i < h->n_tensors; ++i)
        if (strncmp(tensors[i].name, name, sizeof(tensors[i].name)) == 0) return &tensors[i];
    return NULL;
}

#endif /* MB2W_FILE_H */
