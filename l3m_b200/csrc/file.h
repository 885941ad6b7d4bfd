// A mapped, validated .l3m file: header, table of contents, tokenizer, chat template.
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
#include <stddef.h>
#include "l3m_format.h"
#include "tokenizer.h"

typedef struct {
    void             *map;
    size_t            size;
    const l3m_header *h;
    const l3m_tensor *toc;
    l3m_tokenizer     tok;
    int               im_start;       // ChatML, when system is not NULL
    const char       *system;
    uint32_t         *index;          // hashed table-of-contents names (entry + 1; 0 empty)
    uint32_t          index_slots;    // a power of two
} l3m_file;

// 0 on success; otherwise -1 with "l3m: <path>: <reason>" on stderr (the reference's messages,
// src/file.c:14-139, so callers that match on them keep working). Replaces src/file.h:1-22.
int               l3m_file_open(l3m_file *f, const char *path);
void              l3m_file_close(l3m_file *f);
const l3m_tensor *l3m_file_tensor(const l3m_file *f, const char *name);     // NULL if absent
const l3m_tensor *l3m_file_blk(const l3m_file *f, int layer, const char *name);
const void       *l3m_file_data(const l3m_file *f, const l3m_tensor *t);
const float      *l3m_file_f32(const l3m_file *f, const l3m_tensor *t);     // NULL if t is NULL
size_t            l3m_row_bytes(int dtype, int k);    // pack.c

#ifdef __cplusplus
}
#endif
