// The .l3m tokenizer section: a byte-string vocabulary with scores, decoded by table and encoded by
// best-pair merging inside pre-tokenizer pieces. The observable behaviour is the reference's
// (src/tokenizer.c, exercised by its tests/unit/test_tokenizer.py): within a piece, the adjacent
// pair whose concatenation is a vocabulary entry with the highest score merges first, the leftmost
// such pair on equal scores, until no pair merges; an entry's bytes resolve to the highest-scoring
// id carrying them.
//
// Data structures (this file's own):
//   - vocabulary lookup: an open-addressing hash table (FNV-1a over the bytes, linear probing) from
//     byte string to id, built once at init. A candidate pair is looked up without building the
//     concatenated string: the hash runs over the left symbol's bytes, then the right one's.
//   - merging: the symbols of a piece stay at their first positions, linked left and right; a max
//     tournament tree over positions holds, for every live symbol, the score of merging it with its
//     right neighbour (or nothing). The root is the next merge; a merge updates the leaves of the two
//     pairs it changes and removes one, so every step is O(log n) and nothing is ever stale.
#include <stdlib.h>
#include <string.h>
#include "l3m_format.h"
#include "tokenizer.h"

// Longest merged entry the encoder considers (the reference's bound on a merge, with max_len).
#define MERGE_LIMIT 512

static uint32_t fnv_step(uint32_t h, const uint8_t *s, int n) {
    for (int i = 0; i < n; i++) h = (h ^ s[i]) * 16777619u;
    return h;
}
#define FNV_SEED 2166136261u

// The id whose bytes are a[0, na) followed by b[0, nb), or -1.
static int find2(const l3m_tokenizer *t, const uint8_t *a, int na, const uint8_t *b, int nb) {
    const uint32_t mask = t->nslots - 1;
    for (uint32_t i = fnv_step(fnv_step(FNV_SEED, a, na), b, nb) & mask;; i = (i + 1) & mask) {
        const uint32_t e = t->slots[i];
        if (!e) return -1;
        const int id = (int)e - 1, len = t->len[id];
        if (len == na + nb && !memcmp(t->bytes[id], a, (size_t)na) && !memcmp(t->bytes[id] + na, b, (size_t)nb)) return id;
    }
}
static int find(const l3m_tokenizer *t, const uint8_t *s, int n) { return find2(t, s, n, s, 0); }

// Enter id; an entry with the same bytes keeps the higher score (the lower id on equal scores).
static void enter(l3m_tokenizer *t, int id) {
    const uint32_t mask = t->nslots - 1;
    const uint8_t *s = t->bytes[id];
    const int n = t->len[id];
    for (uint32_t i = fnv_step(FNV_SEED, s, n) & mask;; i = (i + 1) & mask) {
        const uint32_t e = t->slots[i];
        if (!e) { t->slots[i] = (uint32_t)id + 1; return; }
        const int old = (int)e - 1;
        if (t->len[old] == n && !memcmp(t->bytes[old], s, (size_t)n)) {
            if (t->score[id] > t->score[old]) t->slots[i] = (uint32_t)id + 1;
            return;
        }
    }
}

int l3m_tokenizer_init(l3m_tokenizer *t, const void *section, size_t size, unsigned flags) {
    memset(t, 0, sizeof *t);
    l3m_tok_header h;
    if (size < sizeof h) return -1;
    memcpy(&h, section, sizeof h);                              // the section need not be aligned
    const size_t avail = size - sizeof h;
    if (h.n_tokens > avail / 6 || (int64_t)h.bos >= (int64_t)h.n_tokens) return -1;   // 6: the smallest entry
    const int n = (int)h.n_tokens;
    t->n = n;
    t->bos = h.bos < 0 ? -1 : h.bos;
    t->eos = h.eos;
    t->max_len = (int)h.max_len;
    t->sp_prefix = (flags & L3M_F_SP_PREFIX) != 0;
    t->digits = (flags & L3M_F_DIGITS) != 0;
    uint32_t ns = 16;
    while (ns < 2u * (uint32_t)n + 16) ns <<= 1;
    t->nslots = ns;
    const uint8_t **bytes = malloc(((size_t)n + 1) * sizeof *bytes);
    uint16_t *lens = malloc(((size_t)n + 1) * sizeof *lens);
    float *score = malloc(((size_t)n + 1) * sizeof *score);
    t->bytes = bytes;
    t->len = lens;
    t->score = score;
    t->slots = calloc(ns, sizeof *t->slots);
    if (!bytes || !lens || !score || !t->slots) { l3m_tokenizer_free(t); return -1; }
    const uint8_t *p = (const uint8_t *)section + sizeof h, *end = (const uint8_t *)section + size;
    for (int i = 0; i < n; i++) {                               // {f32 score, u16 length, bytes}
        if (end - p < 6) { l3m_tokenizer_free(t); return -1; }
        uint16_t len;
        memcpy(&score[i], p, 4);
        memcpy(&len, p + 4, 2);
        if (end - (p + 6) < len) { l3m_tokenizer_free(t); return -1; }
        lens[i] = len;
        bytes[i] = p + 6;
        p += 6 + len;
    }
    for (int i = 0; i < n; i++) enter(t, i);
    // SentencePiece vocabularies split into words at spaces unless some entry spans a word boundary
    // (a space right after a non-space).
    t->sp_words = t->sp_prefix;
    for (int i = 0; i < n && t->sp_words; i++)
        for (int j = 1; j < t->len[i]; j++)
            if (t->bytes[i][j] == ' ' && t->bytes[i][j - 1] != ' ') { t->sp_words = 0; break; }
    return 0;
}

void l3m_tokenizer_free(l3m_tokenizer *t) {
    free((void *)t->bytes);
    free((void *)t->len);
    free((void *)t->score);
    free(t->slots);
    memset(t, 0, sizeof *t);
}

// ---- merging within one piece

typedef struct {
    const l3m_tokenizer *t;
    int32_t *sym;                  // symbol ids, at their first positions; -1 once merged away
    int *right, *left;             // the live neighbours (m: none on the right, -1 on the left)
    int *with;                     // per position: the id its pair with the right neighbour makes, or -1
    int *tree;                     // tournament tree over positions (leaves at size + i): a position or -1
    int m, size;
} merger;

// The better of two positions' pairs: the higher score, the left one on equal scores.
static int better(const merger *g, int a, int b) {
    if (a < 0) return b;
    if (b < 0) return a;
    const float sa = g->t->score[g->with[a]], sb = g->t->score[g->with[b]];
    if (sa != sb) return sa > sb ? a : b;
    return a < b ? a : b;
}

static void leaf_set(merger *g, int i) {
    int id = -1;
    const int r = g->right[i];
    if (g->sym[i] >= 0 && r < g->m) {
        const l3m_tokenizer *t = g->t;
        const int a = g->sym[i], b = g->sym[r], n = t->len[a] + t->len[b];
        if (n <= t->max_len && n <= MERGE_LIMIT) id = find2(t, t->bytes[a], t->len[a], t->bytes[b], t->len[b]);
    }
    g->with[i] = id;
    int k = g->size + i;
    g->tree[k] = id >= 0 ? i : -1;
    for (k >>= 1; k; k >>= 1) g->tree[k] = better(g, g->tree[2 * k], g->tree[2 * k + 1]);
}

// Merge sym[0, m) in place; returns the number of symbols left (packed to the front).
static int merge_piece(const l3m_tokenizer *t, int32_t *sym, int m) {
    if (m < 2) return m;
    merger g = {t, sym, NULL, NULL, NULL, NULL, m, 1};
    while (g.size < m) g.size <<= 1;
    g.right = malloc((size_t)m * sizeof(int));
    g.left = malloc((size_t)m * sizeof(int));
    g.with = malloc((size_t)m * sizeof(int));
    g.tree = malloc(2 * (size_t)g.size * sizeof(int));
    if (!g.right || !g.left || !g.with || !g.tree) {
        free(g.right); free(g.left); free(g.with); free(g.tree);
        return m;
    }
    for (int i = 0; i < 2 * g.size; i++) g.tree[i] = -1;
    for (int i = 0; i < m; i++) { g.right[i] = i + 1; g.left[i] = i - 1; }
    for (int i = 0; i < m; i++) {                               // leaves, then every inner node once
        int id = -1;
        if (i + 1 < m) {
            const int a = sym[i], b = sym[i + 1], n = t->len[a] + t->len[b];
            if (n <= t->max_len && n <= MERGE_LIMIT) id = find2(t, t->bytes[a], t->len[a], t->bytes[b], t->len[b]);
        }
        g.with[i] = id;
        g.tree[g.size + i] = id >= 0 ? i : -1;
    }
    for (int k = g.size - 1; k; k--) g.tree[k] = better(&g, g.tree[2 * k], g.tree[2 * k + 1]);
    for (int i; (i = g.tree[1]) >= 0;) {
        const int r = g.right[i];
        sym[i] = g.with[i];
        sym[r] = -1;
        g.right[i] = g.right[r];
        if (g.right[i] < m) g.left[g.right[i]] = i;
        leaf_set(&g, r);                                        // gone
        leaf_set(&g, i);                                        // its new pair on the right
        if (g.left[i] >= 0) leaf_set(&g, g.left[i]);            // the pair on its left
    }
    int k = 0;
    for (int i = 0; i < m; i++)
        if (sym[i] >= 0) sym[k++] = sym[i];
    free(g.right); free(g.left); free(g.with); free(g.tree);
    return k;
}

// ---- pre-tokenizer

enum { CH_SPACE, CH_LETTER, CH_DIGIT, CH_OTHER };
// Byte classes: ASCII whitespace, ASCII letters and every byte >= 0x80 (UTF-8 text counts as
// letters), ASCII digits, everything else.
static int char_class(uint8_t c) {
    if (c == ' ' || (c >= 9 && c <= 13)) return CH_SPACE;
    if (c >= '0' && c <= '9') return CH_DIGIT;
    if (c >= 0x80 || (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z')) return CH_LETTER;
    return CH_OTHER;
}

static int run_of(const uint8_t *p, int cls) {
    int n = 0;
    while (p[n] && char_class(p[n]) == cls) n++;
    return n;
}

// Length of the piece at p (p non-empty). Byte-level BPE follows GPT-2's pattern, tried in order:
//   's 't 're 've 'm 'll 'd  |  ?letters  |  ?digits  |  ?others  |  spaces not before a non-space  |  spaces
// where a digit stands alone when the vocabulary splits digits (and then takes no space before it).
// SentencePiece: leading spaces plus one word when the vocabulary splits words, else the whole text.
static int piece_len(const l3m_tokenizer *t, const uint8_t *p) {
    if (t->sp_prefix) {
        int n = 0;
        while (p[n] == ' ') n++;
        while (p[n] && !(t->sp_words && p[n] == ' ')) n++;
        return n;
    }
    if (p[0] == '\'') {
        static const char *const tails[] = {"s", "t", "re", "ve", "m", "ll", "d"};
        for (unsigned i = 0; i < sizeof tails / sizeof *tails; i++) {
            const size_t n = strlen(tails[i]);
            if (!strncmp((const char *)p + 1, tails[i], n)) return 1 + (int)n;
        }
    }
    const int c0 = char_class(p[0]);
    if (c0 == CH_DIGIT && t->digits) return 1;
    if (c0 != CH_SPACE) return run_of(p, c0);
    // p[0] is whitespace. A single ' ' joins a following letter, digit (unless digits split) or other run.
    if (p[0] == ' ' && p[1]) {
        const int c1 = char_class(p[1]);
        if (c1 != CH_SPACE && !(c1 == CH_DIGIT && t->digits)) return 1 + run_of(p + 1, c1);
    }
    const int n = run_of(p, CH_SPACE);
    // A run that a non-space follows leaves its last character to the next piece, unless the run is
    // one character or the follower is a split digit (which takes no space).
    if (!p[n] || n == 1 || (t->digits && char_class(p[n]) == CH_DIGIT)) return n;
    return n - 1;
}

// Bytes in the character at p (SentencePiece works on UTF-8 characters): 1 for ASCII, a stray
// continuation byte or a malformed sequence.
static int utf8_char_len(const uint8_t *p) {
    const int n = p[0] < 0x80 ? 1 : p[0] < 0xE0 ? 2 : p[0] < 0xF0 ? 3 : 4;
    for (int i = 1; i < n; i++)
        if ((p[i] & 0xC0) != 0x80) return 1;
    return n;
}

int l3m_tokenizer_encode(const l3m_tokenizer *t, const char *text, int add_bos, int32_t *out, int max) {
    int n = 0;
#define EMIT(id) do { if (n == max) return -1; out[n++] = (id); } while (0)
    if (add_bos && t->bos >= 0) EMIT(t->bos);
    const uint8_t *p = (const uint8_t *)text;
    int start = n;                                               // the first piece merges with the leading space
    if (t->sp_prefix && *p) {                                    // SentencePiece's leading space
        const int sp = find(t, (const uint8_t *)" ", 1);
        if (sp >= 0) EMIT(sp);
    }
    for (; *p; start = n) {
        const int len = piece_len(t, p);
        const uint8_t *end = p + len;
        while (p < end) {                                       // one symbol per character (byte), bytes as a fallback
            const int cl = t->sp_prefix ? utf8_char_len(p) : 1, id = find(t, p, cl);
            if (id >= 0) {
                EMIT(id);
            } else {
                for (int i = 0; i < cl; i++) {
                    const int b = find(t, p + i, 1);
                    if (b >= 0) EMIT(b);
                }
            }
            p += cl;
        }
        n = start + merge_piece(t, out + start, n - start);
    }
#undef EMIT
    return n;
}

const uint8_t *l3m_tokenizer_decode(const l3m_tokenizer *t, int32_t tok, int *len) {
    if (tok < 0 || tok >= t->n) {
        *len = 0;
        return (const uint8_t *)"";
    }
    *len = t->len[tok];
    return t->bytes[tok];
}
