// .l3m reader. The file is mapped read-only and checked once at open, so a malformed file is a clean
// error and never a bad read later; what makes a file valid, and the wording of each complaint, is
// the format's contract (the reference's src/file.c:1-139 and its tests/integration/
// test_robustness.py, which patches files byte by byte and matches on these messages).
//
// This reader's own structure: open runs a fixed sequence of stages over a `reader` (path + the
// file being built), each stage assuming the ones before it passed:
//   map       the file exists, is regular and at least a header long
//   header    magic and version, then the table of contents and tokenizer offsets inside the file
//   entries   every table entry on its own (name, dtype, shape, whole blocks, byte count, extent),
//             then a hashed name index over them (the first entry of a name wins)
//   config    the header's sizes
//   schema    a declarative table of the tensors a configuration calls for (which are required under
//             which flags, their shapes in terms of the configuration, which must be f32), applied
//             to the globals and to every layer; every failure is reported before giving up
//   pairing   the rules across tensors of a layer: wq, wk, wv share a dtype; bq, bk, bv come together
//   tokenizer the tokenizer section, and its size against the vocabulary
//   chat      the optional ChatML section
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include "file.h"

#define SIZE_LIMIT (1u << 24)   // bound on every header size and tensor dimension: products stay in range

typedef struct {
    const char *path;
    l3m_file *f;
} reader;

// Report "l3m: <path>: <message>" and undo the open.
static int reject(reader *r, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "l3m: %s: ", r->path);
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
    l3m_file_close(r->f);
    return -1;
}

// Report without undoing (the schema stage reports every problem, then fails once).
static void complain(const reader *r, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "l3m: %s: ", r->path);
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
}

// ---- the name index: open addressing over the table of contents (entry + 1; 0 = empty)

static uint32_t name_hash(const char *s) {
    uint32_t h = 2166136261u;
    for (int i = 0; i < 64 && s[i]; i++) h = (h ^ (uint8_t)s[i]) * 16777619u;
    return h;
}

static int build_index(l3m_file *f) {
    uint32_t n = 16;
    while (n < 2u * f->h->n_tensors + 16) n <<= 1;
    f->index = calloc(n, sizeof *f->index);
    if (!f->index) return -1;
    f->index_slots = n;
    for (uint32_t i = 0; i < f->h->n_tensors; i++) {
        uint32_t s = name_hash(f->toc[i].name) & (n - 1);
        for (; f->index[s]; s = (s + 1) & (n - 1))
            if (!strncmp(f->toc[f->index[s] - 1].name, f->toc[i].name, sizeof f->toc[i].name)) break;
        if (!f->index[s]) f->index[s] = i + 1;
    }
    return 0;
}

const l3m_tensor *l3m_file_tensor(const l3m_file *f, const char *name) {
    if (!f->index) return NULL;
    const uint32_t mask = f->index_slots - 1;
    for (uint32_t s = name_hash(name) & mask; f->index[s]; s = (s + 1) & mask) {
        const l3m_tensor *t = &f->toc[f->index[s] - 1];
        if (!strncmp(t->name, name, sizeof t->name)) return t;
    }
    return NULL;
}

const l3m_tensor *l3m_file_blk(const l3m_file *f, int layer, const char *name) {
    char full[80];
    snprintf(full, sizeof full, "blk.%d.%s", layer, name);
    return l3m_file_tensor(f, full);
}

const void *l3m_file_data(const l3m_file *f, const l3m_tensor *t) { return (const char *)f->map + t->offset; }

const float *l3m_file_f32(const l3m_file *f, const l3m_tensor *t) { return t ? (const float *)l3m_file_data(f, t) : NULL; }

// ---- stages

static int stage_map(reader *r) {
    l3m_file *f = r->f;
    const int fd = open(r->path, O_RDONLY);
    if (fd < 0) return reject(r, "%s", strerror(errno));
    struct stat st;
    const int usable = !fstat(fd, &st) && S_ISREG(st.st_mode) && (size_t)st.st_size >= sizeof(l3m_header);
    if (!usable) {
        close(fd);
        return reject(r, "not an l3m v%d file", L3M_VERSION);
    }
    f->size = (size_t)st.st_size;
    void *map = mmap(NULL, f->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return reject(r, "mmap: %s", strerror(errno));
    f->map = map;
    f->h = (const l3m_header *)map;
    return 0;
}

static int stage_header(reader *r) {
    l3m_file *f = r->f;
    const l3m_header *h = f->h;
    if (!l3m_header_ok(h)) return reject(r, "not an l3m v%d file", L3M_VERSION);
    const int toc_fits = h->toc_offset % 8 == 0 && h->toc_offset <= f->size &&
                         h->n_tensors <= (f->size - h->toc_offset) / sizeof(l3m_tensor);
    if (!toc_fits || h->tokenizer_offset > f->size) return reject(r, "truncated file");
    f->toc = (const l3m_tensor *)((const char *)f->map + h->toc_offset);
    return 0;
}

// What is wrong with table entry t on its own, or NULL.
static const char *entry_fault(const l3m_file *f, const l3m_tensor *t) {
    if (!memchr(t->name, 0, sizeof t->name)) return "unterminated name";
    if (t->dtype >= L3M_NDTYPES || t->ndim < 1 || t->ndim > 2) return "bad dtype or ndim";
    const uint64_t cols = t->shape[t->ndim - 1], rows = t->ndim == 2 ? t->shape[0] : 1;
    if (rows == 0 || cols == 0 || rows > SIZE_LIMIT || cols > SIZE_LIMIT) return "bad shape";
    const int whole = t->dtype >= L3M_Q8_0 ? cols % L3M_QBLOCK == 0 : t->dtype == L3M_BF16 ? cols % 2 == 0 : 1;
    if (!whole) return "rows are not whole blocks";
    if (t->nbytes != rows * l3m_row_bytes((int)t->dtype, (int)cols)) return "nbytes does not match the shape";
    if (t->offset % 64 || t->offset > f->size || t->nbytes > f->size - t->offset) return "misaligned or past the end of the file";
    return NULL;
}

static int stage_entries(reader *r) {
    l3m_file *f = r->f;
    for (uint32_t i = 0; i < f->h->n_tensors; i++) {
        const char *why = entry_fault(f, &f->toc[i]);
        if (why) return reject(r, "tensor %u (%.64s): %s", i, f->toc[i].name, why);
    }
    if (build_index(f)) return reject(r, "out of memory");
    return 0;
}

static int stage_config(reader *r) {
    const l3m_header *h = r->f->h;
    const uint32_t sizes[] = {h->dim, h->ffn_dim, h->vocab, h->ctx, h->n_layers, h->n_heads, h->n_kv_heads};
    int ok = 1;
    for (unsigned i = 0; i < sizeof sizes / sizeof *sizes; i++) ok &= sizes[i] > 0 && sizes[i] <= SIZE_LIMIT;
    ok = ok && h->dim % h->n_heads == 0 && h->n_heads % h->n_kv_heads == 0 && (h->dim / h->n_heads) % 8 == 0;
    if (!ok)
        return reject(r, "bad config: dim %u, heads %u, kv_heads %u (head_dim a multiple of 8), ffn %u, layers %u, vocab %u, ctx %u", h->dim,
                      h->n_heads, h->n_kv_heads, h->ffn_dim, h->n_layers, h->vocab, h->ctx);
    return 0;
}

// The schema: sizes in terms of the configuration, and when each tensor must be present.
enum size_of { S_NONE, S_DIM, S_KV, S_FFN, S_VOCAB, S_CTX };
enum need { N_ALWAYS, N_OPTIONAL, N_LAYERNORM, N_NOT_GELU, N_NOT_TIED, N_LEARNED_POS };
typedef struct {
    const char *name;
    unsigned char need, f32, rows, cols;       // cols S_NONE: a vector of `rows`
} tensor_rule;

static const tensor_rule kGlobals[] = {
    {"embed", N_ALWAYS, 0, S_VOCAB, S_DIM},      {"lm_head", N_NOT_TIED, 0, S_VOCAB, S_DIM},
    {"pos_embed", N_LEARNED_POS, 1, S_CTX, S_DIM}, {"norm", N_ALWAYS, 1, S_DIM, S_NONE},
    {"norm_b", N_LAYERNORM, 1, S_DIM, S_NONE},
};
static const tensor_rule kPerLayer[] = {
    {"attn_norm", N_ALWAYS, 1, S_DIM, S_NONE}, {"attn_norm_b", N_LAYERNORM, 1, S_DIM, S_NONE},
    {"ffn_norm", N_ALWAYS, 1, S_DIM, S_NONE},  {"ffn_norm_b", N_LAYERNORM, 1, S_DIM, S_NONE},
    {"wq", N_ALWAYS, 0, S_DIM, S_DIM},         {"wk", N_ALWAYS, 0, S_KV, S_DIM},
    {"wv", N_ALWAYS, 0, S_KV, S_DIM},          {"wo", N_ALWAYS, 0, S_DIM, S_DIM},
    {"w_up", N_ALWAYS, 0, S_FFN, S_DIM},       {"w_gate", N_NOT_GELU, 0, S_FFN, S_DIM},
    {"w_down", N_ALWAYS, 0, S_DIM, S_FFN},     {"bo", N_OPTIONAL, 1, S_DIM, S_NONE},
    {"b_up", N_OPTIONAL, 1, S_FFN, S_NONE},    {"b_down", N_OPTIONAL, 1, S_DIM, S_NONE},
    {"bq", N_OPTIONAL, 1, S_DIM, S_NONE},      {"bk", N_OPTIONAL, 1, S_KV, S_NONE},
    {"bv", N_OPTIONAL, 1, S_KV, S_NONE},
};

static uint64_t size_value(const l3m_header *h, int s) {
    switch (s) {
    case S_DIM: return h->dim;
    case S_KV: return (uint64_t)h->dim / h->n_heads * h->n_kv_heads;
    case S_FFN: return h->ffn_dim;
    case S_VOCAB: return h->vocab;
    case S_CTX: return h->ctx;
    default: return 0;
    }
}

static int required(const l3m_header *h, int need) {
    switch (need) {
    case N_ALWAYS: return 1;
    case N_LAYERNORM: return (h->flags & L3M_F_LAYERNORM) != 0;
    case N_NOT_GELU: return (h->flags & L3M_F_GELU) == 0;
    case N_NOT_TIED: return (h->flags & L3M_F_TIED) == 0;
    case N_LEARNED_POS: return (h->flags & L3M_F_LEARNED_POS) != 0;
    default: return 0;
    }
}

// 0 when the rule holds for `name` (present with its shape and dtype, or absent and not required).
static int apply_rule(const reader *r, const tensor_rule *rule, const char *name) {
    const l3m_header *h = r->f->h;
    const l3m_tensor *t = l3m_file_tensor(r->f, name);
    if (!t) {
        if (!required(h, rule->need)) return 0;
        complain(r, "tensor %s missing", name);
        return -1;
    }
    const uint64_t rows = size_value(h, rule->rows), cols = size_value(h, rule->cols);
    const int matrix = rule->cols != S_NONE;
    const int fits = t->ndim == (matrix ? 2u : 1u) && t->shape[0] == rows && (!matrix || t->shape[1] == cols) &&
                     (!rule->f32 || t->dtype == L3M_F32);
    if (fits) return 0;
    char shape[48];
    if (matrix) snprintf(shape, sizeof shape, "[%llu, %llu]", (unsigned long long)rows, (unsigned long long)cols);
    else snprintf(shape, sizeof shape, "[%llu]", (unsigned long long)rows);
    complain(r, "tensor %s: expected %s%s", name, rule->f32 ? "f32 " : "", shape);
    return -1;
}

static int stage_schema(reader *r) {
    const l3m_header *h = r->f->h;
    int faults = 0;
    for (unsigned i = 0; i < sizeof kGlobals / sizeof *kGlobals; i++) faults += apply_rule(r, &kGlobals[i], kGlobals[i].name) != 0;
    char name[80];
    for (uint32_t l = 0; l < h->n_layers; l++)
        for (unsigned i = 0; i < sizeof kPerLayer / sizeof *kPerLayer; i++) {
            snprintf(name, sizeof name, "blk.%u.%s", l, kPerLayer[i].name);
            faults += apply_rule(r, &kPerLayer[i], name) != 0;
        }
    if (faults) {
        l3m_file_close(r->f);
        return -1;
    }
    return 0;
}

// The engine packs a layer's q, k and v rows into one matrix: one dtype, biases all or none.
static int stage_pairing(reader *r) {
    const l3m_file *f = r->f;
    for (uint32_t l = 0; l < f->h->n_layers; l++) {
        const l3m_tensor *q = l3m_file_blk(f, (int)l, "wq"), *k = l3m_file_blk(f, (int)l, "wk"), *v = l3m_file_blk(f, (int)l, "wv");
        const int biases = !!l3m_file_blk(f, (int)l, "bq") + !!l3m_file_blk(f, (int)l, "bk") + !!l3m_file_blk(f, (int)l, "bv");
        if (q->dtype != k->dtype || q->dtype != v->dtype || (biases != 0 && biases != 3))
            return reject(r, "blk.%u: wq, wk, wv must share a dtype, and bq, bk, bv come together", l);
    }
    return 0;
}

static int stage_tokenizer(reader *r) {
    l3m_file *f = r->f;
    const l3m_header *h = f->h;
    if (l3m_tokenizer_init(&f->tok, (const char *)f->map + h->tokenizer_offset, f->size - h->tokenizer_offset, h->flags))
        return reject(r, "bad tokenizer section");
    if (f->tok.n > (int)h->vocab) return reject(r, "tokenizer has %d tokens, vocab only %u", f->tok.n, h->vocab);
    return 0;
}

static int stage_chat(reader *r) {
    l3m_file *f = r->f;
    const uint64_t at = f->h->chat_offset;
    if (!at) return 0;
    l3m_chat_header c;
    if (at > f->size - sizeof c) return reject(r, "bad chat section");
    const char *system = (const char *)f->map + at + sizeof c;
    if (!memchr(system, 0, f->size - at - sizeof c)) return reject(r, "bad chat section");
    memcpy(&c, (const char *)f->map + at, sizeof c);             // the section need not be aligned
    const int in_vocab = c.im_start >= 0 && c.im_start < f->tok.n && f->tok.eos >= 0 && f->tok.eos < f->tok.n;
    if (!in_vocab) return reject(r, "bad chat section");
    f->im_start = c.im_start;
    f->system = system;
    return 0;
}

int l3m_file_open(l3m_file *f, const char *path) {
    memset(f, 0, sizeof *f);
    reader r = {path, f};
    int (*const stages[])(reader *) = {stage_map, stage_header, stage_entries, stage_config, stage_schema,
                                       stage_pairing, stage_tokenizer, stage_chat};
    for (unsigned i = 0; i < sizeof stages / sizeof *stages; i++)
        if (stages[i](&r)) return -1;
    return 0;
}

void l3m_file_close(l3m_file *f) {
    l3m_tokenizer_free(&f->tok);
    free(f->index);
    if (f->map) munmap(f->map, f->size);
    memset(f, 0, sizeof *f);
}
