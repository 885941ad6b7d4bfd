// ORACLE — test infrastructure only (see oracle.h). The decode engine with the scalar kernel table
// on one rank, and the fp32 reference forward, restated from the reference's engine.c and ref.c.
// The reference's sharded engine computes every output on exactly one rank with a fixed order, so
// its logits do not depend on the rank count (reference tests/integration/test_engine.py:217-228):
// one rank is the oracle for every GPU count.
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include "oracle.h"

#define T  O_TILE
#define QB O_QB

enum { F_LAYERNORM = 1, F_LEARNED_POS = 2, F_GELU = 4, F_TIED = 8 };   // reference src/model.h:18-25

typedef struct { const uint8_t *data; int dtype, rows, cols; } tensor;   // rows 1 for vectors

typedef struct { uint8_t *tiles; int ntiles, k, dtype; } shard;

typedef struct {
    shard qkv, wo, up, gate, down;
    const float *bq, *bk, *bv, *bo, *b_up, *b_down, *attn_norm, *attn_norm_b, *ffn_norm, *ffn_norm_b;
    uint16_t *kc, *vc;                                  // [ctx][kv_dim] bf16
    float *wq_f, *wk_f, *wv_f, *wo_f, *up_f, *gate_f, *down_f;   // dequantised, for the fp32 reference
} layer;

struct o_model {
    uint8_t *map; size_t size;
    uint32_t flags; int dim, n_layers, n_heads, n_kv, ffn, vocab, ctx, hd, kv_dim;
    float theta, eps;
    int bos, eos;
    tensor embed, lm_head, pos_embed;
    const float *norm, *norm_b;
    layer *L;
    shard head;
    float *x, *xb, *qkv, *attn, *proj, *h, *gate, *down, *logits;
    void *scratch;
    // fp32 reference state
    float *embed_f, *head_f;
    uint16_t *rkc, *rvc;
    float *rq, *rk, *rv, *ratt, *rhb, *rg, *rlogits;
    int ref_ready;
};

static uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
static uint64_t rd64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }
static float rdf(const uint8_t *p) { float v; memcpy(&v, p, 4); return v; }

// The table of contents: 120-byte entries {name[64], dtype, ndim, shape[4], offset, nbytes}
// (reference src/model.h:39-44).
static int find(const o_model *m, const char *name, tensor *out) {
    uint32_t n = rd32(m->map + 64);
    const uint8_t *toc = m->map + rd64(m->map + 72);
    for (uint32_t i = 0; i < n; i++) {
        const uint8_t *e = toc + (size_t)i * 120;
        if (strncmp((const char *)e, name, 64)) continue;
        out->dtype = (int)rd32(e + 64);
        int ndim = (int)rd32(e + 68);
        out->rows = ndim == 2 ? (int)rd64(e + 72) : 1;
        out->cols = (int)rd64(e + 72 + 8 * (ndim - 1));
        out->data = m->map + rd64(e + 104);
        return 1;
    }
    return 0;
}

static const float *vec(const o_model *m, const char *name) {
    tensor t;
    return find(m, name, &t) ? (const float *)t.data : NULL;
}

static const float *blk_vec(const o_model *m, int l, const char *name) {
    char buf[64];
    snprintf(buf, sizeof buf, "blk.%d.%s", l, name);
    return vec(m, buf);
}

static int blk(const o_model *m, int l, const char *name, tensor *t) {
    char buf[64];
    snprintf(buf, sizeof buf, "blk.%d.%s", l, name);
    return find(m, buf, t);
}

static const void *row_of(const tensor *t, int r) { return t->data + (size_t)r * o_row_bytes(t->dtype, t->cols); }

// Pack rows[0..n) into whole tiles (reference engine.c:110-122): missing rows pack as zeros.
static shard pack_rows(int dtype, int k, const void **rows, int n) {
    shard s = { NULL, (n + T - 1) / T, k, dtype };
    size_t tb = o_tile_bytes(dtype, k);
    s.tiles = aligned_alloc(64, (size_t)s.ntiles * tb + 64);
    for (int t = 0; t < s.ntiles; t++) {
        const void *tr[T];
        for (int j = 0; j < T; j++) tr[j] = t * T + j < n ? rows[t * T + j] : NULL;
        o_pack_tile(s.tiles + (size_t)t * tb, dtype, tr, k);
    }
    return s;
}

static shard pack_tensor(const tensor *t) {
    const void **rows = malloc(sizeof *rows * (size_t)t->rows);
    for (int r = 0; r < t->rows; r++) rows[r] = row_of(t, r);
    shard s = pack_rows(t->dtype, t->cols, rows, t->rows);
    free(rows);
    return s;
}

o_model *o_load(const char *path, int ctx) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) { perror(path); return NULL; }
    struct stat st;
    fstat(fd, &st);
    o_model *m = calloc(1, sizeof *m);
    m->size = (size_t)st.st_size;
    m->map = mmap(NULL, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m->map == MAP_FAILED || m->size < 1024 || memcmp(m->map, "l3m", 3)) { fprintf(stderr, "oracle: %s: not an l3m file\n", path); free(m); return NULL; }
    const uint8_t *h = m->map;
    m->flags = rd32(h + 24); m->dim = (int)rd32(h + 28); m->n_layers = (int)rd32(h + 32); m->n_heads = (int)rd32(h + 36);
    m->n_kv = (int)rd32(h + 40); m->ffn = (int)rd32(h + 44); m->vocab = (int)rd32(h + 48);
    int hctx = (int)rd32(h + 52);
    m->theta = rdf(h + 56); m->eps = rdf(h + 60);
    m->hd = m->dim / m->n_heads; m->kv_dim = m->hd * m->n_kv;
    int want = ctx > 0 ? ctx : 512;
    m->ctx = hctx < want ? hctx : want;                  // reference engine.c:435
    const uint8_t *tok = m->map + rd64(h + 80);
    m->bos = (int32_t)rd32(tok + 4); m->eos = (int32_t)rd32(tok + 8);
    if (m->bos < 0) m->bos = -1;

    find(m, "embed", &m->embed);
    if (!find(m, (m->flags & F_TIED) ? "embed" : "lm_head", &m->lm_head)) { fprintf(stderr, "oracle: no lm_head\n"); return NULL; }
    if (m->flags & F_LEARNED_POS) find(m, "pos_embed", &m->pos_embed);
    m->norm = vec(m, "norm"); m->norm_b = vec(m, "norm_b");
    m->L = calloc((size_t)m->n_layers, sizeof *m->L);
    int nqkv = m->dim + 2 * m->kv_dim;
    const void **rows = malloc(sizeof *rows * (size_t)nqkv);
    for (int l = 0; l < m->n_layers; l++) {
        layer *L = &m->L[l];
        tensor wq, wk, wv, t;
        blk(m, l, "wq", &wq); blk(m, l, "wk", &wk); blk(m, l, "wv", &wv);
        // q rows of every head, then k rows, then v rows (reference engine.c:135-152 on one rank).
        for (int r = 0; r < m->dim; r++) rows[r] = row_of(&wq, r);
        for (int r = 0; r < m->kv_dim; r++) rows[m->dim + r] = row_of(&wk, r);
        for (int r = 0; r < m->kv_dim; r++) rows[m->dim + m->kv_dim + r] = row_of(&wv, r);
        L->qkv = pack_rows(wq.dtype, m->dim, rows, nqkv);
        blk(m, l, "wo", &t); L->wo = pack_tensor(&t);
        blk(m, l, "w_up", &t); L->up = pack_tensor(&t);
        if (!(m->flags & F_GELU)) { blk(m, l, "w_gate", &t); L->gate = pack_tensor(&t); }
        blk(m, l, "w_down", &t); L->down = pack_tensor(&t);
        L->bq = blk_vec(m, l, "bq"); L->bk = blk_vec(m, l, "bk"); L->bv = blk_vec(m, l, "bv"); L->bo = blk_vec(m, l, "bo");
        L->b_up = blk_vec(m, l, "b_up"); L->b_down = blk_vec(m, l, "b_down");
        L->attn_norm = blk_vec(m, l, "attn_norm"); L->attn_norm_b = blk_vec(m, l, "attn_norm_b");
        L->ffn_norm = blk_vec(m, l, "ffn_norm"); L->ffn_norm_b = blk_vec(m, l, "ffn_norm_b");
        L->kc = calloc((size_t)m->ctx * m->kv_dim, 2);
        L->vc = calloc((size_t)m->ctx * m->kv_dim, 2);
    }
    free(rows);
    m->head = pack_tensor(&m->lm_head);
    int big = m->ffn > m->dim ? m->ffn : m->dim;
    m->x = calloc((size_t)m->dim, 4); m->xb = calloc((size_t)m->dim, 4); m->attn = calloc((size_t)m->dim, 4);
    m->proj = calloc((size_t)m->dim + T, 4); m->down = calloc((size_t)m->dim + T, 4);
    m->qkv = calloc((size_t)nqkv + T, 4); m->h = calloc((size_t)m->ffn + T, 4); m->gate = calloc((size_t)m->ffn + T, 4);
    m->logits = calloc((size_t)m->head.ntiles * T, 4);
    m->scratch = calloc((size_t)2 * big + 64, 1);
    return m;
}

int o_vocab(const o_model *m) { return m->vocab; }
int o_ctx(const o_model *m) { return m->ctx; }
int o_eos(const o_model *m) { return m->eos; }
int o_bos(const o_model *m) { return m->bos; }

static void add(float *x, const float *y, int n) { for (int i = 0; i < n; i++) x[i] += y[i]; }

// reference src/ops.c:20-27: sequential mean; sequential variance, its squares rounded on their own
// over the part of the row the reference build vectorises (o_rmsnorm_fused_from, as in rmsnorm) and fused into
// the sum in the tail; then (d*s)*w + b as one fma.
void o_layernorm(float *y, const float *x, const float *w, const float *b, int n, float eps) {
    float mean = 0.0f, var = 0.0f;
    for (int i = 0; i < n; i++) mean += x[i];
    mean /= (float)n;
    const int split = o_rmsnorm_fused_from(n);
    for (int i = 0; i < n; i++) {
        const float d = x[i] - mean;
        if (i < split) { const float sq = d * d; var += sq; }
        else var = fmaf(d, d, var);
    }
    float s = 1.0f / sqrtf(var / (float)n + eps);
    for (int i = 0; i < n; i++) y[i] = fmaf((x[i] - mean) * s, w[i], b[i]);
}

// reference src/ops.c:53-56 (tanh approximation): x + 0.044715 x^3 contracts to one fma.
void o_gelu(float *x, int n) {
    for (int i = 0; i < n; i++) {
        float v = x[i];
        float inner = fmaf((0.044715f * v) * v, v, v);
        x[i] = (0.5f * v) * (1.0f + tanhf(0.7978845608f * inner));
    }
}

static void norm(const o_model *m, float *y, const float *x, const float *w, const float *b) {
    if (m->flags & F_LAYERNORM) o_layernorm(y, x, w, b, m->dim, m->eps);
    else o_rmsnorm(y, x, w, m->dim, m->eps);
}

// reference engine.c:219-223
static void gemv(o_model *m, float *y, const shard *s, const float *x) {
    o_vec v;
    o_vec_prepare(&v, s->dtype, x, s->k, m->scratch);
    o_gemv(s->dtype, y, s->tiles, s->ntiles, s->k, &v);
}

// reference engine.c:230-281 with one rank: every head, every tile.
const float *o_forward(o_model *m, int32_t tok, int pos, int want_logits) {
    int dim = m->dim, hd = m->hd, kvd = m->kv_dim, hpk = m->n_heads / m->n_kv;
    o_dequant_row(m->x, m->embed.dtype, row_of(&m->embed, tok), dim);
    if (m->pos_embed.data) add(m->x, (const float *)row_of(&m->pos_embed, pos), dim);
    for (int l = 0; l < m->n_layers; l++) {
        layer *L = &m->L[l];
        norm(m, m->xb, m->x, L->attn_norm, L->attn_norm_b);
        float *q = m->qkv, *k = q + dim, *v = k + kvd;
        gemv(m, q, &L->qkv, m->xb);
        if (L->bq) { add(q, L->bq, dim); add(k, L->bk, kvd); add(v, L->bv, kvd); }
        if (!(m->flags & F_LEARNED_POS)) { o_rope(q, m->n_heads, hd, pos, m->theta); o_rope(k, m->n_kv, hd, pos, m->theta); }
        uint16_t *kc = L->kc + (size_t)pos * kvd, *vc = L->vc + (size_t)pos * kvd;
        for (int i = 0; i < kvd; i++) { kc[i] = o_f32_to_bf16(k[i]); vc[i] = o_f32_to_bf16(v[i]); }
        for (int j = 0; j < m->n_heads; j++)
            o_attend(m->attn + j * hd, q + j * hd, L->kc + (j / hpk) * hd, L->vc + (j / hpk) * hd, pos, hd, kvd);

        gemv(m, m->proj, &L->wo, m->attn);
        if (L->bo) add(m->proj, L->bo, dim);
        add(m->x, m->proj, dim);

        norm(m, m->xb, m->x, L->ffn_norm, L->ffn_norm_b);
        gemv(m, m->h, &L->up, m->xb);
        if (L->b_up) add(m->h, L->b_up, m->ffn);
        if (m->flags & F_GELU) o_gelu(m->h, m->ffn);
        else { gemv(m, m->gate, &L->gate, m->xb); o_silu_mul(m->h, m->gate, m->ffn); }

        gemv(m, m->down, &L->down, m->h);
        if (L->b_down) add(m->down, L->b_down, dim);
        add(m->x, m->down, dim);
    }
    if (!want_logits) return NULL;
    norm(m, m->xb, m->x, m->norm, m->norm_b);
    gemv(m, m->logits, &m->head, m->xb);
    return m->logits;
}

// ---- fp32 reference forward (reference src/ref.c:24-143)

static float *dequant_matrix(const tensor *t) {
    float *out = malloc((size_t)t->rows * t->cols * 4);
    for (int r = 0; r < t->rows; r++) o_dequant_row(out + (size_t)r * t->cols, t->dtype, row_of(t, r), t->cols);
    return out;
}

// reference ref.c:35-42: out[i] = Σ_j w[i][j] x[j] in input order, then + bias. As in the f32
// kernel, the compiler vectorises the products 8 (then 4) wide and adds them one by one; the
// inputs past o_rmsnorm_fused_from(k) each take one fused multiply-add.
static void matvec(float *out, const float *w, const float *x, const float *bias, int n, int k) {
    int split = o_rmsnorm_fused_from(k);
    for (int i = 0; i < n; i++) {
        const float *r = w + (size_t)i * k;
        float acc = 0.0f;
        for (int j = 0; j < split; j++) acc = acc + r[j] * x[j];
        for (int j = split; j < k; j++) acc = fmaf(r[j], x[j], acc);
        out[i] = acc + (bias ? bias[i] : 0.0f);
    }
}

static void ref_prepare(o_model *m) {
    if (m->ref_ready) return;
    tensor t;
    m->embed_f = dequant_matrix(&m->embed);
    m->head_f = (m->flags & F_TIED) ? m->embed_f : dequant_matrix(&m->lm_head);
    for (int l = 0; l < m->n_layers; l++) {
        layer *L = &m->L[l];
        blk(m, l, "wq", &t); L->wq_f = dequant_matrix(&t);
        blk(m, l, "wk", &t); L->wk_f = dequant_matrix(&t);
        blk(m, l, "wv", &t); L->wv_f = dequant_matrix(&t);
        blk(m, l, "wo", &t); L->wo_f = dequant_matrix(&t);
        blk(m, l, "w_up", &t); L->up_f = dequant_matrix(&t);
        if (!(m->flags & F_GELU)) { blk(m, l, "w_gate", &t); L->gate_f = dequant_matrix(&t); }
        blk(m, l, "w_down", &t); L->down_f = dequant_matrix(&t);
    }
    size_t kv = (size_t)m->n_layers * m->ctx * m->kv_dim;
    m->rkc = calloc(kv, 2); m->rvc = calloc(kv, 2);
    m->rq = calloc((size_t)m->dim, 4); m->ratt = calloc((size_t)m->dim, 4);
    m->rk = calloc((size_t)m->kv_dim, 4); m->rv = calloc((size_t)m->kv_dim, 4);
    m->rhb = calloc((size_t)m->ffn, 4); m->rg = calloc((size_t)m->ffn, 4);
    m->rlogits = calloc((size_t)m->vocab, 4);
    m->ref_ready = 1;
}

const float *o_ref_forward(o_model *m, int32_t tok, int pos) {
    ref_prepare(m);
    int dim = m->dim, ffn = m->ffn, hd = m->hd, kvd = m->kv_dim, hpk = m->n_heads / m->n_kv;
    float *x = m->x, *xb = m->xb;
    memcpy(x, m->embed_f + (size_t)tok * dim, (size_t)dim * 4);
    if (m->pos_embed.data) add(x, (const float *)row_of(&m->pos_embed, pos), dim);
    for (int l = 0; l < m->n_layers; l++) {
        layer *L = &m->L[l];
        norm(m, xb, x, L->attn_norm, L->attn_norm_b);
        matvec(m->rq, L->wq_f, xb, L->bq, dim, dim);
        matvec(m->rk, L->wk_f, xb, L->bk, kvd, dim);
        matvec(m->rv, L->wv_f, xb, L->bv, kvd, dim);
        if (!(m->flags & F_LEARNED_POS)) { o_rope(m->rq, m->n_heads, hd, pos, m->theta); o_rope(m->rk, m->n_kv, hd, pos, m->theta); }
        uint16_t *kc = m->rkc + ((size_t)l * m->ctx + pos) * kvd, *vc = m->rvc + ((size_t)l * m->ctx + pos) * kvd;
        for (int i = 0; i < kvd; i++) { kc[i] = o_f32_to_bf16(m->rk[i]); vc[i] = o_f32_to_bf16(m->rv[i]); }
        for (int j = 0; j < m->n_heads; j++) {
            size_t off = (size_t)l * m->ctx * kvd + (size_t)(j / hpk) * hd;
            o_attend(m->ratt + j * hd, m->rq + j * hd, m->rkc + off, m->rvc + off, pos, hd, kvd);
        }
        matvec(xb, L->wo_f, m->ratt, L->bo, dim, dim);
        add(x, xb, dim);
        norm(m, xb, x, L->ffn_norm, L->ffn_norm_b);
        matvec(m->rhb, L->up_f, xb, L->b_up, ffn, dim);
        if (m->flags & F_GELU) o_gelu(m->rhb, ffn);
        else { matvec(m->rg, L->gate_f, xb, NULL, ffn, dim); o_silu_mul(m->rhb, m->rg, ffn); }
        matvec(xb, L->down_f, m->rhb, L->b_down, dim, ffn);
        add(x, xb, dim);
    }
    norm(m, xb, x, m->norm, m->norm_b);
    matvec(m->rlogits, m->head_f, xb, NULL, m->vocab, dim);
    return m->rlogits;
}

// reference engine.c:290-301 (greedy): first maximum wins (strict >), starting below every value.
static int32_t argmax(const float *logits, int n) {
    float mx = -INFINITY; int32_t idx = 0;
    for (int i = 0; i < n; i++) if (logits[i] > mx) { mx = logits[i]; idx = i; }
    return idx;
}

// reference engine.c:98-101: xorshift64*, a double in [0, 1).
static double rand01(uint64_t *s) {
    *s ^= *s >> 12;
    *s ^= *s << 25;
    *s ^= *s >> 27;
    return (double)((*s * 0x2545F4914F6CDD1DULL) >> 11) * (1.0 / 9007199254740992.0);
}

// reference engine.c:283-287: the unnormalised weight of a logit, 0 below e^-16 of the maximum.
static float prob(float logit, float gmax, float temp) {
    float d = (logit - gmax) / temp;
    return d < -16 ? 0 : o_expf(d);
}

// reference engine.c:370-384 (and 290-330 with one rank): the greedy choice when temp is not > 0;
// else the first index whose running double sum of weights exceeds u * z (z the whole sum, u the
// next draw), the last index when none does (a NaN sum).
int32_t o_sample(const float *logits, int n, float temp, uint64_t *rng) {
    float gmax = -INFINITY;
    int32_t best = 0;
    for (int i = 0; i < n; i++) if (logits[i] > gmax) { gmax = logits[i]; best = i; }
    if (!(temp > 0)) return best;
    float *probs = malloc((size_t)n * sizeof(float));
    double z = 0;
    for (int i = 0; i < n; i++) z += probs[i] = prob(logits[i], gmax, temp);
    double target = rand01(rng) * z, c = 0;
    int32_t tok = n - 1;
    for (int i = 0; i < n; i++) if ((c += probs[i]) > target) { tok = i; break; }
    free(probs);
    return tok;
}

// reference engine.c:322-327, 342-362 (and 364-386 for the reference path), temperature 0.
int o_generate(o_model *m, const int32_t *prompt, int n_prompt, int max_new, int32_t *out, float *logits_out,
               int *n_pos, int reference) {
    return o_generate_t(m, prompt, n_prompt, max_new, 0.0f, 0, out, logits_out, n_pos, reference);
}

// The same with temperature sampling (reference engine.c:549-555 seeds the generator).
int o_generate_t(o_model *m, const int32_t *prompt, int n_prompt, int max_new, float temp, uint64_t seed, int32_t *out,
                 float *logits_out, int *n_pos, int reference) {
    uint64_t rng = seed * 0x9E3779B97F4A7C15ULL + 1;
    if (n_prompt < 1 || n_prompt >= m->ctx) { if (n_pos) *n_pos = 0; return 0; }
    int n_gen = 0, pos = 0, rows = 0;
    int32_t tok = 0;
    for (;; pos++) {
        int last = pos >= n_prompt - 1;
        if (pos < n_prompt) tok = prompt[pos];
        int stop = last && (n_gen >= max_new || pos + 1 >= m->ctx);
        const float *lg;
        if (reference) {
            lg = o_ref_forward(m, tok, pos);
            if (!last) continue;
        } else {
            lg = o_forward(m, tok, pos, last);
            if (!last) continue;
        }
        if (logits_out) memcpy(logits_out + (size_t)rows * m->vocab, lg, (size_t)m->vocab * 4);
        rows++;
        if (stop) break;
        tok = temp > 0 ? o_sample(lg, m->vocab, temp, &rng) : argmax(lg, m->vocab);
        if (tok == m->eos || tok == m->bos) break;
        out[n_gen++] = tok;
    }
    if (n_pos) *n_pos = pos + 1;
    return n_gen;
}

void o_free(o_model *m) {
    if (!m) return;
    for (int l = 0; l < m->n_layers; l++) {
        layer *L = &m->L[l];
        free(L->qkv.tiles); free(L->wo.tiles); free(L->up.tiles); free(L->gate.tiles); free(L->down.tiles);
        free(L->kc); free(L->vc);
        free(L->wq_f); free(L->wk_f); free(L->wv_f); free(L->wo_f); free(L->up_f); free(L->gate_f); free(L->down_f);
    }
    free(m->L); free(m->head.tiles);
    if (m->head_f != m->embed_f) free(m->head_f);
    free(m->embed_f); free(m->rkc); free(m->rvc); free(m->rq); free(m->rk); free(m->rv); free(m->ratt); free(m->rhb); free(m->rg); free(m->rlogits);
    free(m->x); free(m->xb); free(m->attn); free(m->proj); free(m->down); free(m->qkv); free(m->h); free(m->gate); free(m->logits); free(m->scratch);
    munmap(m->map, m->size);
    free(m);
}
