// Greedy merge tokenizer: repeatedly merge the adjacent pair whose concatenation is a token with the
// highest score (leftmost on ties), within pre-tokenizer pieces. Semantics follow the reference
// (src/tokenizer.c:1-177; SentencePiece scores as in llama2.c, -rank for byte-level BPE); the merge
// loop here is a priority queue over candidate pairs with lazy invalidation, O(n log n) per piece.
#include <stdlib.h>
#include <string.h>
#include "l3m_format.h"
#include "tokenizer.h"

static const l3m_tokenizer *sort_ctx;   // qsort has no context argument in C11

static int cmp_bytes(const uint8_t *a, int na, const uint8_t *b, int nb) {
    int c = memcmp(a, b, (size_t)(na < nb ? na : nb));
    return c ? c : na - nb;
}

static int order_cmp(const void *pa, const void *pb) {
    const l3m_tokenizer *t = sort_ctx;
    int a = *(const int *)pa, b = *(const int *)pb;
    int c = cmp_bytes(t->bytes[a], t->len[a], t->bytes[b], t->len[b]);
    if (c) return c;
    if (t->score[a] != t->score[b]) return t->score[a] > t->score[b] ? -1 : 1;
    return a - b;
}

int l3m_tokenizer_init(l3m_tokenizer *t, const void *section, size_t size, unsigned flags) {
    memset(t, 0, sizeof *t);
    l3m_tok_header h;
    if (size < sizeof h) return -1;
    memcpy(&h, section, sizeof h);
    if (h.n_tokens > (size - sizeof h) / 6 || h.bos >= (int64_t)h.n_tokens) return -1;
    t->n = (int)h.n_tokens;
    t->bos = h.bos < 0 ? -1 : h.bos;
    t->eos = h.eos;
    t->max_len = (int)h.max_len;
    t->sp_prefix = (flags & L3M_F_SP_PREFIX) != 0;
    t->digits = (flags & L3M_F_DIGITS) != 0;
    size_t m = (size_t)t->n + 1;
    const uint8_t **bytes = malloc(m * sizeof *bytes);
    uint16_t *len = malloc(m * sizeof *len);
    float *score = malloc(m * sizeof *score);
    t->order = malloc(m * sizeof *t->order);
    t->bytes = bytes; t->len = len; t->score = score;
    if (!bytes || !len || !score || !t->order) { l3m_tokenizer_free(t); return -1; }
    const uint8_t *p = (const uint8_t *)section + sizeof h, *end = (const uint8_t *)section + size;
    for (int i = 0; i < t->n; i++) {
        if (end - p < 6) { l3m_tokenizer_free(t); return -1; }
        memcpy(&score[i], p, 4);
        memcpy(&len[i], p + 4, 2);
        if (end - p - 6 < len[i]) { l3m_tokenizer_free(t); return -1; }
        bytes[i] = p + 6;
        p += 6 + len[i];
        t->order[i] = i;
    }
    // SentencePiece words: a piece is a word with its leading spaces, unless some token has a space
    // after a non-space (then the whole text is one piece).
    t->sp_words = t->sp_prefix;
    for (int i = 0; i < t->n && t->sp_words; i++)
        for (int j = 1; j < len[i]; j++)
            if (bytes[i][j] == ' ' && bytes[i][j - 1] != ' ') t->sp_words = 0;
    sort_ctx = t;
    qsort(t->order, (size_t)t->n, sizeof *t->order, order_cmp);
    return 0;
}

void l3m_tokenizer_free(l3m_tokenizer *t) {
    free((void *)t->bytes); free((void *)t->len); free((void *)t->score); free(t->order);
    memset(t, 0, sizeof *t);
}

// The id whose bytes are exactly s[0..n), the highest-scored among duplicates; -1 if none.
static int lookup(const l3m_tokenizer *t, const uint8_t *s, int n) {
    int lo = 0, hi = t->n;
    while (lo < hi) {
        int mid = (lo + hi) / 2, id = t->order[mid];
        if (cmp_bytes(t->bytes[id], t->len[id], s, n) < 0) lo = mid + 1; else hi = mid;
    }
    if (lo == t->n) return -1;
    int id = t->order[lo];
    return cmp_bytes(t->bytes[id], t->len[id], s, n) == 0 ? id : -1;
}

// ---- merging inside one piece

typedef struct { float score; int left, right, a, b, id; } cand;

static int cand_before(const cand *x, const cand *y) {
    return x->score > y->score || (x->score == y->score && x->left < y->left);
}

typedef struct { cand *v; int n; } heap;

static void heap_push(heap *h, cand c) {
    int i = h->n++;
    while (i > 0 && cand_before(&c, &h->v[(i - 1) / 2])) { h->v[i] = h->v[(i - 1) / 2]; i = (i - 1) / 2; }
    h->v[i] = c;
}

static cand heap_pop(heap *h) {
    cand top = h->v[0], last = h->v[--h->n];
    int i = 0;
    for (;;) {
        int c = 2 * i + 1;
        if (c >= h->n) break;
        if (c + 1 < h->n && cand_before(&h->v[c + 1], &h->v[c])) c++;
        if (!cand_before(&h->v[c], &last)) break;
        h->v[i] = h->v[c];
        i = c;
    }
    h->v[i] = last;
    return top;
}

static void offer(const l3m_tokenizer *t, heap *h, const int32_t *s, int left, int right) {
    uint8_t buf[1024];
    int a = s[left], b = s[right], n = t->len[a] + t->len[b];
    if (n > t->max_len || n > (int)sizeof buf) return;
    memcpy(buf, t->bytes[a], t->len[a]);
    memcpy(buf + t->len[a], t->bytes[b], t->len[b]);
    int id = lookup(t, buf, n);
    if (id >= 0) heap_push(h, (cand){t->score[id], left, right, a, b, id});
}

// Merge out[lo, n) in place; returns the new n.
static int merge_piece(const l3m_tokenizer *t, int32_t *out, int lo, int n) {
    int m = n - lo;
    if (m < 2) return n;
    int32_t *s = out + lo;
    int *next = malloc((size_t)m * sizeof *next), *prev = malloc((size_t)m * sizeof *prev);
    heap h = {malloc((size_t)3 * m * sizeof(cand)), 0};       // m - 1 initial pairs, at most two more per merge
    if (!next || !prev || !h.v) { free(next); free(prev); free(h.v); return n; }
    for (int i = 0; i < m; i++) { next[i] = i + 1; prev[i] = i - 1; }
    for (int i = 0; i + 1 < m; i++) offer(t, &h, s, i, i + 1);
    while (h.n) {
        cand c = heap_pop(&h);
        if (next[c.left] != c.right || s[c.left] != c.a || s[c.right] != c.b) continue;   // stale
        s[c.left] = c.id;
        s[c.right] = -1;
        next[c.left] = next[c.right];
        if (next[c.left] < m) prev[next[c.left]] = c.left;
        if (prev[c.left] >= 0) offer(t, &h, s, prev[c.left], c.left);
        if (next[c.left] < m) offer(t, &h, s, c.left, next[c.left]);
    }
    int k = 0;
    for (int i = 0; i < m; i++) if (s[i] >= 0) s[k++] = s[i];
    free(next); free(prev); free(h.v);
    return lo + k;
}

// ---- pre-tokenizer

enum { C_SPACE, C_LETTER, C_DIGIT, C_PUNCT };

static int char_class(uint8_t c) {                 // non-ASCII counts as a letter
    if (c == ' ' || (c >= '\t' && c <= '\r')) return C_SPACE;
    if (c >= '0' && c <= '9') return C_DIGIT;
    if (c >= 0x80 || ((c | 32) >= 'a' && (c | 32) <= 'z')) return C_LETTER;
    return C_PUNCT;
}

static int utf8_len(const uint8_t *p) {
    int n = p[0] < 0x80 ? 1 : p[0] < 0xE0 ? 2 : p[0] < 0xF0 ? 3 : 4;
    for (int i = 1; i < n; i++)
        if ((p[i] & 0xC0) != 0x80) return 1;
    return n;
}

// End of the piece starting at p. Byte-level BPE follows GPT-2's pre-tokenizer:
//   's|'t|'re|'ve|'m|'ll|'d| ?letters| ?digits| ?other| spaces not before a word | spaces
// with single digits when t->digits. SentencePiece: a word with its leading spaces if sp_words,
// else the rest of the text.
static const uint8_t *piece_end(const l3m_tokenizer *t, const uint8_t *p) {
    if (t->sp_prefix) {
        while (*p == ' ') p++;
        while (*p && (*p != ' ' || !t->sp_words)) p++;
        return p;
    }
    static const char *const contractions[] = {"s", "t", "re", "ve", "m", "ll", "d"};
    if (*p == '\'')
        for (int i = 0; i < 7; i++) {
            size_t n = strlen(contractions[i]);
            if (!strncmp((const char *)p + 1, contractions[i], n)) return p + 1 + n;
        }
    if (t->digits && char_class(*p) == C_DIGIT) return p + 1;
    const uint8_t *q = p;
    if (*p == ' ' && p[1] && char_class(p[1]) != C_SPACE && !(t->digits && char_class(p[1]) == C_DIGIT)) q++;
    int k = char_class(*q);
    if (k != C_SPACE) {
        while (*q && char_class(*q) == k) q++;
        return q;
    }
    while (*q && char_class(*q) == C_SPACE) q++;
    int at_end = !*q || (t->digits && char_class(*q) == C_DIGIT);
    return (q - p > 1 && !at_end) ? q - 1 : q;       // the last space goes to the next word
}

int l3m_tokenizer_encode(const l3m_tokenizer *t, const char *text, int add_bos, int32_t *out, int max) {
    int n = 0;
    if (add_bos && t->bos >= 0) {
        if (n == max) return -1;
        out[n++] = t->bos;
    }
    int lo = n, space = lookup(t, (const uint8_t *)" ", 1);
    if (t->sp_prefix && *text && space >= 0) {
        if (n == max) return -1;
        out[n++] = space;
    }
    for (const uint8_t *p = (const uint8_t *)text; *p; lo = n) {
        const uint8_t *end = piece_end(t, p);
        while (p < end) {
            int len = t->sp_prefix ? utf8_len(p) : 1, id = lookup(t, p, len);
            if (id >= 0) {
                if (n == max) return -1;
                out[n++] = id;
            } else {
                for (int i = 0; i < len; i++)                 // byte fallback
                    if ((id = lookup(t, p + i, 1)) >= 0) {
                        if (n == max) return -1;
                        out[n++] = id;
                    }
            }
            p += len;
        }
        n = merge_piece(t, out, lo, n);
    }
    return n;
}

const uint8_t *l3m_tokenizer_decode(const l3m_tokenizer *t, int32_t tok, int *len) {
    if (tok < 0 || tok >= t->n) { *len = 0; return (const uint8_t *)""; }
    *len = t->len[tok];
    return t->bytes[tok];
}
