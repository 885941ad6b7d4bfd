// .l3m reader. Everything is checked once at open, so a malformed file is a clean error and never a
// bad read later (the reference's contract, src/file.c:1-139; tests/integration/test_robustness.py
// patches files byte by byte and expects these messages).
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include "file.h"

#define DIM_LIMIT (1u << 24)   // every header size and tensor dimension stays below this

static int fail(l3m_file *f, const char *path, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "l3m: %s: ", path);
    vfprintf(stderr, fmt, ap);
    fputc('\n', stderr);
    va_end(ap);
    l3m_file_close(f);
    return -1;
}

// What is wrong with one table-of-contents entry, or NULL.
static const char *entry_problem(const l3m_file *f, const l3m_tensor *t) {
    if (!memchr(t->name, 0, sizeof t->name)) return "unterminated name";
    if (t->dtype >= L3M_NDTYPES || t->ndim < 1 || t->ndim > 2) return "bad dtype or ndim";
    uint64_t rows = t->ndim == 2 ? t->shape[0] : 1, cols = t->shape[t->ndim - 1];
    if (rows == 0 || cols == 0 || rows > DIM_LIMIT || cols > DIM_LIMIT) return "bad shape";
    int quantised = t->dtype >= L3M_Q8_0;
    if ((quantised && cols % L3M_QBLOCK) || (t->dtype == L3M_BF16 && cols % 2)) return "rows are not whole blocks";
    if (t->nbytes != rows * l3m_row_bytes((int)t->dtype, (int)cols)) return "nbytes does not match the shape";
    if (t->offset % 64 || t->offset > f->size || t->nbytes > f->size - t->offset) return "misaligned or past the end of the file";
    return NULL;
}

// 1 present and well shaped, 0 absent and optional, -1 an error (reported). cols 0: a vector.
static int expect(const l3m_file *f, const char *path, const char *name, int required, int must_f32, uint64_t rows, uint64_t cols) {
    const l3m_tensor *t = l3m_file_tensor(f, name);
    if (!t) {
        if (required) fprintf(stderr, "l3m: %s: tensor %s missing\n", path, name);
        return required ? -1 : 0;
    }
    int ok = t->ndim == (cols ? 2u : 1u) && t->shape[0] == rows && (!cols || t->shape[1] == cols) && (!must_f32 || t->dtype == L3M_F32);
    if (ok) return 1;
    if (cols) fprintf(stderr, "l3m: %s: tensor %s: expected %s[%llu, %llu]\n", path, name, must_f32 ? "f32 " : "",
                      (unsigned long long)rows, (unsigned long long)cols);
    else fprintf(stderr, "l3m: %s: tensor %s: expected %s[%llu]\n", path, name, must_f32 ? "f32 " : "", (unsigned long long)rows);
    return -1;
}

static int check_config(const l3m_file *f, const char *path) {
    const l3m_header *h = f->h;
    int bad = !h->dim || !h->ffn_dim || !h->vocab || !h->ctx || !h->n_layers || !h->n_heads || !h->n_kv_heads ||
              h->dim > DIM_LIMIT || h->ffn_dim > DIM_LIMIT || h->vocab > DIM_LIMIT || h->ctx > DIM_LIMIT || h->n_layers > DIM_LIMIT;
    if (!bad) bad = h->dim % h->n_heads || h->n_heads % h->n_kv_heads || (h->dim / h->n_heads) % 8;
    if (bad)
        fprintf(stderr, "l3m: %s: bad config: dim %u, heads %u, kv_heads %u (head_dim a multiple of 8), ffn %u, layers %u, vocab %u, ctx %u\n",
                path, h->dim, h->n_heads, h->n_kv_heads, h->ffn_dim, h->n_layers, h->vocab, h->ctx);
    return bad ? -1 : 0;
}

static int check_tensors(const l3m_file *f, const char *path) {
    const l3m_header *h = f->h;
    uint32_t d = h->dim, F = h->ffn_dim, V = h->vocab, kv = h->dim / h->n_heads * h->n_kv_heads;
    int ln = (h->flags & L3M_F_LAYERNORM) != 0, gelu = (h->flags & L3M_F_GELU) != 0, err = 0;
    err |= expect(f, path, "embed", 1, 0, V, d) < 0;
    if (!(h->flags & L3M_F_TIED)) err |= expect(f, path, "lm_head", 1, 0, V, d) < 0;
    err |= expect(f, path, "pos_embed", (h->flags & L3M_F_LEARNED_POS) != 0, 1, h->ctx, d) < 0;
    err |= expect(f, path, "norm", 1, 1, d, 0) < 0;
    err |= expect(f, path, "norm_b", ln, 1, d, 0) < 0;
    if (err) return -1;
    char n[80];
    for (uint32_t l = 0; l < h->n_layers; l++) {
#define NAME(s) (snprintf(n, sizeof n, "blk.%u.%s", l, s), n)
        err |= expect(f, path, NAME("attn_norm"), 1, 1, d, 0) < 0;
        err |= expect(f, path, NAME("attn_norm_b"), ln, 1, d, 0) < 0;
        err |= expect(f, path, NAME("ffn_norm"), 1, 1, d, 0) < 0;
        err |= expect(f, path, NAME("ffn_norm_b"), ln, 1, d, 0) < 0;
        err |= expect(f, path, NAME("wq"), 1, 0, d, d) < 0;
        err |= expect(f, path, NAME("wk"), 1, 0, kv, d) < 0;
        err |= expect(f, path, NAME("wv"), 1, 0, kv, d) < 0;
        err |= expect(f, path, NAME("wo"), 1, 0, d, d) < 0;
        err |= expect(f, path, NAME("w_up"), 1, 0, F, d) < 0;
        err |= expect(f, path, NAME("w_gate"), !gelu, 0, F, d) < 0;
        err |= expect(f, path, NAME("w_down"), 1, 0, d, F) < 0;
        err |= expect(f, path, NAME("bo"), 0, 1, d, 0) < 0;
        err |= expect(f, path, NAME("b_up"), 0, 1, F, 0) < 0;
        err |= expect(f, path, NAME("b_down"), 0, 1, d, 0) < 0;
        int bq = expect(f, path, NAME("bq"), 0, 1, d, 0);
        int bk = expect(f, path, NAME("bk"), 0, 1, kv, 0);
        int bv = expect(f, path, NAME("bv"), 0, 1, kv, 0);
#undef NAME
        if (err || bq < 0 || bk < 0 || bv < 0) return -1;
        const l3m_tensor *q = l3m_file_blk(f, (int)l, "wq"), *k = l3m_file_blk(f, (int)l, "wk"), *v = l3m_file_blk(f, (int)l, "wv");
        if (bq != bk || bq != bv || k->dtype != q->dtype || v->dtype != q->dtype) {   // packed as one shard per head
            fprintf(stderr, "l3m: %s: blk.%u: wq, wk, wv must share a dtype, and bq, bk, bv come together\n", path, l);
            return -1;
        }
    }
    return 0;
}

int l3m_file_open(l3m_file *f, const char *path) {
    memset(f, 0, sizeof *f);
    int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(f, path, "%s", strerror(errno));
    struct stat st;
    if (fstat(fd, &st) || !S_ISREG(st.st_mode) || (size_t)st.st_size < sizeof(l3m_header)) {
        close(fd);
        return fail(f, path, "not an l3m v%d file", L3M_VERSION);
    }
    f->size = (size_t)st.st_size;
    void *map = mmap(NULL, f->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) return fail(f, path, "mmap: %s", strerror(errno));
    f->map = map;
    f->h = (const l3m_header *)map;
    const l3m_header *h = f->h;
    if (!l3m_header_ok(h)) return fail(f, path, "not an l3m v%d file", L3M_VERSION);
    if (h->toc_offset % 8 || h->toc_offset > f->size || h->n_tensors > (f->size - h->toc_offset) / sizeof(l3m_tensor) ||
        h->tokenizer_offset > f->size)
        return fail(f, path, "truncated file");
    f->toc = (const l3m_tensor *)((const char *)map + h->toc_offset);
    for (uint32_t i = 0; i < h->n_tensors; i++) {
        const char *why = entry_problem(f, &f->toc[i]);
        if (why) return fail(f, path, "tensor %u (%.64s): %s", i, f->toc[i].name, why);
    }
    if (check_config(f, path) || check_tensors(f, path)) { l3m_file_close(f); return -1; }
    if (l3m_tokenizer_init(&f->tok, (const char *)map + h->tokenizer_offset, f->size - h->tokenizer_offset, h->flags))
        return fail(f, path, "bad tokenizer section");
    if (f->tok.n > (int)h->vocab) return fail(f, path, "tokenizer has %d tokens, vocab only %u", f->tok.n, h->vocab);
    if (h->chat_offset) {
        l3m_chat_header c;
        if (h->chat_offset > f->size - sizeof c) return fail(f, path, "bad chat section");
        const char *sys = (const char *)map + h->chat_offset + sizeof c;
        if (!memchr(sys, 0, f->size - h->chat_offset - sizeof c)) return fail(f, path, "bad chat section");
        memcpy(&c, (const char *)map + h->chat_offset, sizeof c);
        if (c.im_start < 0 || c.im_start >= f->tok.n || f->tok.eos < 0 || f->tok.eos >= f->tok.n) return fail(f, path, "bad chat section");
        f->im_start = c.im_start;
        f->system = sys;
    }
    return 0;
}

void l3m_file_close(l3m_file *f) {
    l3m_tokenizer_free(&f->tok);
    if (f->map) munmap(f->map, f->size);
    memset(f, 0, sizeof *f);
}

const l3m_tensor *l3m_file_tensor(const l3m_file *f, const char *name) {
    for (uint32_t i = 0; i < f->h->n_tensors; i++)
        if (!strncmp(f->toc[i].name, name, sizeof f->toc[i].name)) return &f->toc[i];
    return NULL;
}

const l3m_tensor *l3m_file_blk(const l3m_file *f, int layer, const char *name) {
    char buf[80];
    snprintf(buf, sizeof buf, "blk.%d.%s", layer, name);
    return l3m_file_tensor(f, buf);
}

const void *l3m_file_data(const l3m_file *f, const l3m_tensor *t) { return (const char *)f->map + t->offset; }

const float *l3m_file_f32(const l3m_file *f, const l3m_tensor *t) { return t ? (const float *)l3m_file_data(f, t) : NULL; }
