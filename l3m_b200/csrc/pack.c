// Host side of the tile layout: row and tile sizes, packing file rows into 16-output tiles,
// dequantising a row, and preparing an activation (bf16, or q8 with per-32 scale and sum).
// Byte-for-byte the reference's layout and arithmetic (src/pack.c:10-122), so tiles packed here and
// by the reference are interchangeable. Built with -ffp-contract=off: every expression rounds as written.
#include <math.h>
#include <string.h>
#include "l3m_format.h"
#include "numerics.h"
#include "../../include/l3m_kernels.h"

#define T  L3M_TILE
#define QB L3M_QBLOCK

size_t l3m_row_bytes(int dtype, int k) {
    switch (dtype) {
    case L3M_F32:   return (size_t)k * 4;
    case L3M_BF16:  return (size_t)k * 2;
    case L3M_Q8_0:  return (size_t)(k / QB) * sizeof(l3m_block_q8_0);
    case L3M_Q4_0:  return (size_t)(k / QB) * sizeof(l3m_block_q4_0);
    case L3M_MXFP4: return (size_t)(k / QB) * sizeof(l3m_block_mxfp4);
    }
    return 0;
}

size_t l3m_tile_bytes(int dtype, int k) {
    switch (dtype) {
    case L3M_F32:   return (size_t)k * T * 4;
    case L3M_BF16:  return (size_t)k * T * 2;
    case L3M_Q8_0:  return (size_t)(k / QB) * (2 * T + QB * T);
    case L3M_Q4_0:  return (size_t)(k / QB) * (2 * T + QB * T / 2);
    case L3M_MXFP4: return (size_t)(k / QB) * (T + QB * T / 2);
    }
    return 0;
}

// Element i of a ggml 4-bit block as its nibble (low nibbles hold 0..15, high ones 16..31).
static int nibble(const uint8_t *qs, int i) { return i < 16 ? (qs[i] & 15) : (qs[i - 16] >> 4); }

void l3m_pack_tile(void *dst, int dtype, const void *const rows[T], int k) {
    memset(dst, 0, l3m_tile_bytes(dtype, k));
    if (dtype == L3M_F32) {
        float *w = dst;
        for (int c = 0; c < T; c++)
            if (rows[c]) for (int i = 0; i < k; i++) w[(size_t)i * T + c] = ((const float *)rows[c])[i];
        return;
    }
    if (dtype == L3M_BF16) {
        uint16_t *w = dst;
        for (int c = 0; c < T; c++)
            if (rows[c]) for (int i = 0; i < k; i++) w[((size_t)(i / 2) * T + c) * 2 + i % 2] = ((const uint16_t *)rows[c])[i];
        return;
    }
    size_t bb = l3m_tile_bytes(dtype, QB), sb = dtype == L3M_MXFP4 ? T : 2 * T, rb = l3m_row_bytes(dtype, QB);
    for (int b = 0; b < k / QB; b++) {
        uint8_t *blk = (uint8_t *)dst + (size_t)b * bb, *q = blk + sb;
        for (int c = 0; c < T; c++) {
            if (!rows[c]) continue;
            const uint8_t *src = (const uint8_t *)rows[c] + (size_t)b * rb;
            if (dtype == L3M_Q8_0) {
                memcpy(blk + 2 * c, src, 2);
                for (int i = 0; i < QB; i++) q[(i / 4 * T + c) * 4 + i % 4] = (uint8_t)((int8_t)src[2 + i] + 128);
                continue;
            }
            const uint8_t *qs;
            if (dtype == L3M_Q4_0) { memcpy(blk + 2 * c, src, 2); qs = src + 2; }
            else { blk[c] = src[0]; qs = src + 1; }
            for (int g = 0; g < 4; g++)
                for (int j = 0; j < 4; j++) q[(g * T + c) * 4 + j] = (uint8_t)(nibble(qs, 8 * g + j) | nibble(qs, 8 * g + 4 + j) << 4);
        }
    }
}

void l3m_dequant_row(float *out, int dtype, const void *row, int k) {
    const uint8_t *r = row;
    if (dtype == L3M_F32) { memcpy(out, row, (size_t)k * 4); return; }
    if (dtype == L3M_BF16) {
        for (int i = 0; i < k; i++) { uint16_t h; memcpy(&h, r + 2 * i, 2); out[i] = l3m_bf16_to_f32(h); }
        return;
    }
    size_t rb = l3m_row_bytes(dtype, QB);
    for (int b = 0; b < k / QB; b++) {
        const uint8_t *blk = r + (size_t)b * rb;
        float d;
        if (dtype == L3M_MXFP4) d = l3m_e8m0_half(blk[0]);
        else { uint16_t h; memcpy(&h, blk, 2); d = l3m_f16_to_f32(h); }
        for (int i = 0; i < QB; i++) {
            int q = dtype == L3M_Q8_0 ? (int8_t)blk[2 + i]
                  : dtype == L3M_Q4_0 ? nibble(blk + 2, i) - 8 : l3m_mxfp4_value(nibble(blk + 1, i));
            out[b * QB + i] = d * (float)q;
        }
    }
}

void l3m_vec_prepare(l3m_vec *v, int dtype, const float *x, int n, void *scratch) {
    v->f32 = x; v->bf16 = NULL; v->q8 = NULL; v->scale = NULL; v->sum = NULL;
    if (dtype == L3M_F32) return;
    if (dtype == L3M_BF16) {
        uint16_t *h = scratch;
        for (int i = 0; i < n; i++) h[i] = l3m_f32_to_bf16(x[i]);
        v->bf16 = h;
        return;
    }
    int8_t *q = scratch;
    float *scale = (float *)(q + n);
    int32_t *sum = (int32_t *)(scale + n / QB);
    for (int b = 0; b < n / QB; b++) {
        const float *xb = x + b * QB;
        float amax = 0.0f;
        for (int i = 0; i < QB; i++) amax = fabsf(xb[i]) > amax ? fabsf(xb[i]) : amax;
        float inv = amax > 0 ? 127.0f / amax : 0.0f;
        int32_t s = 0;
        for (int i = 0; i < QB; i++) s += q[b * QB + i] = (int8_t)(int)rintf(xb[i] * inv);
        scale[b] = amax / 127.0f;
        sum[b] = s;
    }
    v->q8 = q; v->scale = scale; v->sum = sum;
}
