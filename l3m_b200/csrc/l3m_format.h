// The .l3m v1 on-disk format, as the loader reads it. The layout is the reference's format (fpedd/l3m
// src/model.h:3-70) — it has to be, since the files are the input — restated here field by field.
//
//   [header 1024 B][tensors, each 64-byte aligned][table of contents][tokenizer][chat, optional]
//   Matrices are [rows = outputs][cols = inputs], row-major, quantised in blocks of 32 inputs (ggml).
#pragma once
#include <stdint.h>
#ifdef __cplusplus
#define L3M_STATIC_ASSERT static_assert
#else
#define L3M_STATIC_ASSERT _Static_assert
#endif

#define L3M_VERSION 1
#define L3M_QBLOCK  32            // inputs per quantisation block
#define L3M_TILE    16            // outputs per packed tile

enum l3m_dtype { L3M_F32, L3M_BF16, L3M_Q8_0, L3M_Q4_0, L3M_MXFP4, L3M_NDTYPES };

static inline const char *l3m_dtype_name(int dtype) {
    static const char *names[L3M_NDTYPES] = {"f32", "bf16", "q8_0", "q4_0", "mxfp4"};
    return dtype >= 0 && dtype < L3M_NDTYPES ? names[dtype] : "?";
}

enum l3m_flags {                  // reference src/model.h:18-25
    L3M_F_LAYERNORM   = 1 << 0,   // LayerNorm with bias tensors, else RMSNorm
    L3M_F_LEARNED_POS = 1 << 1,   // pos_embed tensor, else adjacent-pair RoPE
    L3M_F_GELU        = 1 << 2,   // MLP is gelu_tanh(up), else silu(gate) * up
    L3M_F_TIED        = 1 << 3,   // lm_head is the embed tensor
    L3M_F_SP_PREFIX   = 1 << 4,   // SentencePiece tokenizer: prepend a space
    L3M_F_DIGITS      = 1 << 5,   // byte-level BPE: split every digit off
};

typedef struct {                  // reference src/model.h:27-37
    char     magic[4];            // "l3m\0"
    uint32_t version;
    char     arch[16];
    uint32_t flags;
    uint32_t dim, n_layers, n_heads, n_kv_heads, ffn_dim, vocab, ctx;
    float    rope_theta, norm_eps;
    uint32_t n_tensors, reserved;
    uint64_t toc_offset, tokenizer_offset, chat_offset;
    uint8_t  pad[1024 - 96];
} l3m_header;
L3M_STATIC_ASSERT(sizeof(l3m_header) == 1024, "header is 1024 bytes");

typedef struct {                  // reference src/model.h:39-44
    char     name[64];
    uint32_t dtype, ndim;
    uint64_t shape[4];
    uint64_t offset, nbytes;
} l3m_tensor;
L3M_STATIC_ASSERT(sizeof(l3m_tensor) == 120, "toc entries are 120 bytes");

typedef struct { uint32_t n_tokens; int32_t bos, eos; uint32_t max_len; } l3m_tok_header;   // then {f32 score, u16 len, bytes}
typedef struct { int32_t im_start; } l3m_chat_header;                                         // then the system prompt, NUL-ended

// ggml blocks (reference src/model.h:58-60)
typedef struct { uint16_t d; int8_t  qs[32]; } l3m_block_q8_0;    // x = q * d
typedef struct { uint16_t d; uint8_t qs[16]; } l3m_block_q4_0;    // nibble i: low = x[i], high = x[i+16]; x = (q - 8) * d
typedef struct { uint8_t  e; uint8_t qs[16]; } l3m_block_mxfp4;   // same nibbles; x = lut[q] * 2^(e-127) / 2

static inline int l3m_header_ok(const l3m_header *h) {
    return h->magic[0] == 'l' && h->magic[1] == '3' && h->magic[2] == 'm' && h->version == L3M_VERSION;
}
