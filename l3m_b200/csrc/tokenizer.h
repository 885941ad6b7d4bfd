// The tokenizer section of a .l3m file: byte-table decoder and best-pair merge encoder, with the
// reference's observable behaviour (src/tokenizer.h:1-19 is the interface this replaces).
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
#include <stddef.h>
#include <stdint.h>

typedef struct {
    int             n, bos, eos, max_len;     // bos -1: none
    int             sp_prefix, sp_words, digits;
    const uint8_t **bytes;                    // into the file mapping
    const uint16_t *len;
    const float    *score;
    uint32_t       *slots;                    // hash table bytes -> id + 1 (0: empty), nslots a power of two
    uint32_t        nslots;
} l3m_tokenizer;

int            l3m_tokenizer_init(l3m_tokenizer *t, const void *section, size_t size, unsigned flags);   // -1 if malformed
void           l3m_tokenizer_free(l3m_tokenizer *t);
// Token count, or -1 when the ids before merging do not fit in max.
int            l3m_tokenizer_encode(const l3m_tokenizer *t, const char *text, int add_bos, int32_t *out, int max);
const uint8_t *l3m_tokenizer_decode(const l3m_tokenizer *t, int32_t tok, int *len);   // not NUL-terminated

#ifdef __cplusplus
}
#endif
