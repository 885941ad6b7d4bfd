// ORACLE — test infrastructure only. A plain-C restatement of the reference's (fpedd/l3m) scalar
// decode path, used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
// checker. The product (l3m_b200) never links, loads or calls anything here.
//
// Every floating-point expression is written with explicit fmaf() where the reference's compiler
// (gcc -O3 -march=x86-64-v3 -ffp-contract=fast, reference Makefile:2) forms a fused multiply-add,
// and this file is compiled with -ffp-contract=off, so the arithmetic is pinned in the source.
// tests/test_oracle.py checks every function bit-for-bit against the reference compiled from its
// own sources (oracle/_ref/libl3m_all.so) and against the reference's golden vectors.
#pragma once
#include <stddef.h>
#include <stdint.h>

#define O_TILE 16
#define O_QB   32
enum { O_F32, O_BF16, O_Q8_0, O_Q4_0, O_MXFP4, O_NDTYPES };

// ---- conversions (reference src/ops.h:5-6, src/ops.c:5-11)
float    o_bf16_to_f32(uint16_t h);
uint16_t o_f32_to_bf16(float f);
float    o_f16_to_f32(uint16_t h);

// ---- tile layout (reference src/pack.c:10-30, 55-99, 101-122)
size_t o_row_bytes(int dtype, int k);
size_t o_tile_bytes(int dtype, int k);
void   o_pack_tile(void *dst, int dtype, const void *const rows[O_TILE], int k);
void   o_dequant_row(float *out, int dtype, const void *row, int k);
// The prepared activation: bf16 copy, or q8 with per-32 scale and sum (reference src/kernels.h:24-30).
typedef struct { const float *f32; uint16_t *bf16; int8_t *q8; float *scale; int32_t *sum; } o_vec;
void   o_vec_prepare(o_vec *v, int dtype, const float *x, int n, void *scratch);   // scratch >= 2n + 8n/32 bytes

// ---- scalar kernels (reference src/kernels_scalar.c:9-75)
void o_gemv(int dtype, float *y, const void *tiles, int ntiles, int k, const o_vec *x);
// Per-block exact integer dots, block-major: dots[(t*16 + c) * (k/32) + b] = sum_i w*q_x with the
// dtype's offset already removed (the value the reference converts to float in its epilogue).
void o_block_dots(int dtype, int32_t *dots, const void *tiles, int ntiles, int k, const o_vec *x);
// Unpacked integer weights and block scales of a tile set: q[(t*16+c)*k + i], d[(t*16+c)*(k/32) + b].
void o_unpack(int dtype, int8_t *q, float *d, const void *tiles, int ntiles, int k);

// ---- per-token ops (reference src/ops.c:13-73)
void o_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
int  o_rmsnorm_fused_from(int n);   // first index whose square is added by fma (see oracle_kernels.c)
void o_rope(float *v, int n_heads, int head_dim, int pos, float theta);
void o_silu_mul(float *h, const float *gate, int n);
void o_attend(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int head_dim, int stride);

// ---- the engine forward with the scalar table, on one rank (reference src/engine.c:219-281, 290-301,
// 342-362). Logits are bit-identical across the reference's rank counts, so one rank is the oracle.
typedef struct o_model o_model;
o_model     *o_load(const char *path, int ctx);        // NULL on failure, message on stderr
void         o_free(o_model *m);
int          o_vocab(const o_model *m);
int          o_ctx(const o_model *m);
int          o_eos(const o_model *m);
int          o_bos(const o_model *m);
// Feed one token at pos; when want_logits, return the logits (vocab floats, owned by the model).
const float *o_forward(o_model *m, int32_t tok, int pos, int want_logits);
// The fp32 reference forward (reference src/ref.c:98-143): no activation quantisation.
const float *o_ref_forward(o_model *m, int32_t tok, int pos);
// Greedy generate (reference engine.c:342-362 with temperature 0): writes up to max_new tokens to
// out and, when logits_out is not NULL, the logits of every position that sampled ([n][vocab]).
// Returns the number generated; *n_pos gets the positions run (prompt included).
int          o_generate(o_model *m, const int32_t *prompt, int n_prompt, int max_new, int32_t *out,
                        float *logits_out, int *n_pos, int reference);
// The same with temperature sampling (temp > 0; seed as l3m_generate's).
int          o_generate_t(o_model *m, const int32_t *prompt, int n_prompt, int max_new, float temp, uint64_t seed,
                          int32_t *out, float *logits_out, int *n_pos, int reference);
// One draw of the reference's sampler over logits[0..n) (reference engine.c:283-287, 370-384):
// argmax when temp is not > 0; advances *rng only when it samples.
int32_t      o_sample(const float *logits, int n, float temp, uint64_t *rng);

// reference src/ops.c:20-27 and 53-56, exposed so tests can compare them with the reference's.
void o_layernorm(float *y, const float *x, const float *w, const float *b, int n, float eps);
void o_gelu(float *x, int n);

// ---- libm expf, as the reference calls it (softmax, SiLU); exposed so tests can compare.
float o_expf(float x);
// The correctly rounded double evaluation used to build the GPU's exception list: returns the
// double approximation of e^x; see oracle_expf.c.
void o_expf_n(const float *x, float *y, int n);
