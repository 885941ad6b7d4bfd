// ORACLE — test infrastructure only (see oracle.h). Scalar kernels, tile packing and per-token ops,
// restated from the reference with explicit fmaf() at each place its compiler contracts.
#include <math.h>
#include <string.h>
#include "oracle.h"

#define T  O_TILE
#define QB O_QB

typedef union { float f; uint32_t u; } fbits;

// reference src/ops.h:5 — bf16 is the top half of an fp32.
float o_bf16_to_f32(uint16_t h) { fbits v; v.u = (uint32_t)h << 16; return v.f; }

// reference src/ops.h:6 — round to nearest even on the dropped 16 bits (no NaN special case).
uint16_t o_f32_to_bf16(float f) {
    fbits v; v.f = f;
    uint32_t lsb = (v.u >> 16) & 1u;
    return (uint16_t)((v.u + 0x7FFFu + lsb) >> 16);
}

// reference src/ops.c:5-11 — binary16 to binary32, subnormals through ldexpf, inf/NaN kept.
float o_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        float mag = ldexpf((float)m, -24);
        return sign ? -mag : mag;
    }
    fbits v;
    v.u = e == 31 ? (sign | 0x7F800000u | m << 13) : (sign | (e + 112u) << 23 | m << 13);
    return v.f;
}

// Bytes per block of 32 inputs in a 16-output tile: scales then quants (reference pack.c:21-30).
static size_t tile_block_bytes(int dtype) {
    switch (dtype) {
    case O_Q8_0:  return 2 * T + QB * T;
    case O_Q4_0:  return 2 * T + QB * T / 2;
    case O_MXFP4: return T + QB * T / 2;
    }
    return 0;
}

// reference src/pack.c:10-19 (ggml block sizes: q8_0 34, q4_0 18, mxfp4 17 bytes per 32 inputs).
size_t o_row_bytes(int dtype, int k) {
    switch (dtype) {
    case O_F32:   return (size_t)k * 4;
    case O_BF16:  return (size_t)k * 2;
    case O_Q8_0:  return (size_t)(k / QB) * 34;
    case O_Q4_0:  return (size_t)(k / QB) * 18;
    case O_MXFP4: return (size_t)(k / QB) * 17;
    }
    return 0;
}

size_t o_tile_bytes(int dtype, int k) {
    if (dtype == O_F32) return (size_t)k * T * 4;
    if (dtype == O_BF16) return (size_t)k * T * 2;
    return (size_t)(k / QB) * tile_block_bytes(dtype);
}

// Element i of a ggml 4-bit block as its nibble: low nibbles hold 0..15, high nibbles 16..31.
static int nibble_at(const uint8_t *qs, int i) { return i < 16 ? (qs[i] & 15) : (qs[i - 16] >> 4); }

static const int8_t MX_LUT[16]   = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};   // doubled e2m1
static const int8_t MX_LUT16[16] = {16, 17, 18, 19, 20, 22, 24, 28, 16, 15, 14, 13, 12, 10, 8, 4};

// reference src/pack.c:64-99 — interleave 16 file rows into one tile; a NULL row packs as zeros.
void o_pack_tile(void *dst, int dtype, const void *const rows[T], int k) {
    memset(dst, 0, o_tile_bytes(dtype, k));
    if (dtype == O_F32 || dtype == O_BF16) {
        for (int c = 0; c < T; c++) {
            if (!rows[c]) continue;
            for (int i = 0; i < k; i++) {
                if (dtype == O_F32) ((float *)dst)[(size_t)i * T + c] = ((const float *)rows[c])[i];
                else ((uint16_t *)dst)[((size_t)(i >> 1) * T + c) * 2 + (i & 1)] = ((const uint16_t *)rows[c])[i];
            }
        }
        return;
    }
    size_t bb = tile_block_bytes(dtype), row_block = o_row_bytes(dtype, QB), sb = dtype == O_MXFP4 ? T : 2 * T;
    for (int b = 0; b < k / QB; b++) {
        uint8_t *blk = (uint8_t *)dst + (size_t)b * bb, *q = blk + sb;
        for (int c = 0; c < T; c++) {
            if (!rows[c]) continue;
            const uint8_t *src = (const uint8_t *)rows[c] + (size_t)b * row_block;
            if (dtype == O_MXFP4) blk[c] = src[0];
            else memcpy(blk + 2 * c, src, 2);
            const uint8_t *qs = src + (dtype == O_MXFP4 ? 1 : 2);
            if (dtype == O_Q8_0) {
                for (int i = 0; i < QB; i++) q[((i >> 2) * T + c) * 4 + (i & 3)] = (uint8_t)((int8_t)qs[i] + 128);
            } else {
                for (int g = 0; g < 4; g++)
                    for (int j = 0; j < 4; j++)
                        q[(g * T + c) * 4 + j] = (uint8_t)(nibble_at(qs, 8 * g + j) | nibble_at(qs, 8 * g + 4 + j) << 4);
            }
        }
    }
}

// Scale of block b of a file row (reference pack.c:35-42): f16, or 2^(e-128) for e8m0.
static float row_block_scale(int dtype, const uint8_t *row, int b) {
    const uint8_t *blk = row + (size_t)b * o_row_bytes(dtype, QB);
    if (dtype == O_MXFP4) return ldexpf(1.0f, (int)blk[0] - 128);
    uint16_t d; memcpy(&d, blk, 2);
    return o_f16_to_f32(d);
}

static int row_block_q(int dtype, const uint8_t *row, int b, int i) {
    const uint8_t *blk = row + (size_t)b * o_row_bytes(dtype, QB);
    if (dtype == O_Q8_0) return (int8_t)blk[2 + i];
    if (dtype == O_Q4_0) return nibble_at(blk + 2, i) - 8;
    return MX_LUT[nibble_at(blk + 1, i)];
}

// reference src/pack.c:55-62
void o_dequant_row(float *out, int dtype, const void *row, int k) {
    const uint8_t *r = row;
    if (dtype == O_F32) { memcpy(out, row, (size_t)k * 4); return; }
    if (dtype == O_BF16) {
        for (int i = 0; i < k; i++) { uint16_t h; memcpy(&h, r + 2 * i, 2); out[i] = o_bf16_to_f32(h); }
        return;
    }
    for (int b = 0; b < k / QB; b++) {
        float d = row_block_scale(dtype, r, b);
        for (int i = 0; i < QB; i++) out[b * QB + i] = d * (float)row_block_q(dtype, r, b, i);
    }
}

// reference src/pack.c:101-122 — bf16 by RNE; q8 per 32: inv = 127/amax, q = rint(x*inv),
// scale = amax/127, sum = Σq. scratch layout as the reference: q8[n], scale[n/32], sum[n/32].
void o_vec_prepare(o_vec *v, int dtype, const float *x, int n, void *scratch) {
    v->f32 = x; v->bf16 = NULL; v->q8 = NULL; v->scale = NULL; v->sum = NULL;
    if (dtype == O_F32) return;
    if (dtype == O_BF16) {
        v->bf16 = scratch;
        for (int i = 0; i < n; i++) v->bf16[i] = o_f32_to_bf16(x[i]);
        return;
    }
    v->q8 = scratch;
    v->scale = (float *)(v->q8 + n);
    v->sum = (int32_t *)(v->scale + n / QB);
    for (int b = 0; b < n / QB; b++) {
        const float *xb = x + b * QB;
        float amax = 0.0f;
        for (int i = 0; i < QB; i++) { float a = fabsf(xb[i]); if (a > amax) amax = a; }
        float inv = amax > 0 ? 127.0f / amax : 0.0f;
        int32_t s = 0;
        for (int i = 0; i < QB; i++) {
            int8_t q = (int8_t)(int)rintf(xb[i] * inv);
            v->q8[b * QB + i] = q;
            s += q;
        }
        v->scale[b] = amax / 127.0f;
        v->sum[b] = s;
    }
}

// ---- the integer part of each quantised kernel: exact dots per (output, block)

// The weight of output c, input i of block b in a quantised tile, as the stored (offset) integer.
static int tile_q_raw(int dtype, const uint8_t *blk, int c, int i, int *offset) {
    size_t sb = dtype == O_MXFP4 ? T : 2 * T;
    const uint8_t *q = blk + sb;
    if (dtype == O_Q8_0) { *offset = 128; return q[((i >> 2) * T + c) * 4 + (i & 3)]; }
    int g = i >> 3, j = i & 7;
    uint8_t byte = q[(g * T + c) * 4 + (j & 3)];
    int nib = j < 4 ? (byte & 15) : (byte >> 4);
    if (dtype == O_Q4_0) { *offset = 8; return nib; }
    *offset = 16;
    return MX_LUT16[nib];
}

static float tile_block_scale(int dtype, const uint8_t *blk, int c) {
    if (dtype == O_MXFP4) return ldexpf(1.0f, (int)blk[c] - 128);
    uint16_t d; memcpy(&d, blk + 2 * c, 2);
    return o_f16_to_f32(d);
}

// acc_i - offset * sum_x of the reference's quantised kernels (kernels_scalar.c:37-43, 57-71): exact.
static int32_t block_dot(int dtype, const uint8_t *blk, int c, const int8_t *xq, int32_t xsum) {
    int32_t acc = 0; int offset = 0;
    for (int i = 0; i < QB; i++) acc += tile_q_raw(dtype, blk, c, i, &offset) * (int32_t)xq[i];
    return acc - offset * xsum;
}

void o_block_dots(int dtype, int32_t *dots, const void *tiles, int ntiles, int k, const o_vec *x) {
    size_t tb = o_tile_bytes(dtype, k), bb = tile_block_bytes(dtype);
    int nb = k / QB;
    for (int t = 0; t < ntiles; t++)
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = (const uint8_t *)tiles + t * tb + b * bb;
            for (int c = 0; c < T; c++)
                dots[((size_t)t * T + c) * nb + b] = block_dot(dtype, blk, c, x->q8 + b * QB, x->sum[b]);
        }
}

void o_unpack(int dtype, int8_t *q, float *d, const void *tiles, int ntiles, int k) {
    size_t tb = o_tile_bytes(dtype, k), bb = tile_block_bytes(dtype);
    int nb = k / QB;
    for (int t = 0; t < ntiles; t++)
        for (int b = 0; b < nb; b++) {
            const uint8_t *blk = (const uint8_t *)tiles + t * tb + b * bb;
            for (int c = 0; c < T; c++) {
                size_t o = (size_t)t * T + c;
                d[o * nb + b] = tile_block_scale(dtype, blk, c);
                for (int i = 0; i < QB; i++) {
                    int offset = 0, raw = tile_q_raw(dtype, blk, c, i, &offset);
                    q[o * k + b * QB + i] = (int8_t)(raw - offset);
                }
            }
        }
}

// reference src/kernels_scalar.c:9-75. Per output: the fp32 accumulator runs over the inputs in
// order (f32: rounded product then add, fused at the tail; bf16: exact product, one rounding) or over the blocks in
// order (quantised: the scale product rounds, then one fused multiply-add).
void o_gemv(int dtype, float *y, const void *tiles, int ntiles, int k, const o_vec *x) {
    size_t tb = o_tile_bytes(dtype, k);
    for (int t = 0; t < ntiles; t++) {
        const uint8_t *tile = (const uint8_t *)tiles + t * tb;
        for (int c = 0; c < T; c++) {
            float acc = 0.0f;
            if (dtype == O_F32) {
                const float *w = (const float *)tile;
                // As the squares of o_rmsnorm: inputs before the split add a rounded product, the
                // rest fuse (the compiler vectorises the input loop 8, then 4, wide).
                int split = o_rmsnorm_fused_from(k);
                for (int i = 0; i < split; i++) acc = acc + w[(size_t)i * T + c] * x->f32[i];
                for (int i = split; i < k; i++) acc = fmaf(w[(size_t)i * T + c], x->f32[i], acc);
            } else if (dtype == O_BF16) {
                const uint16_t *w = (const uint16_t *)tile;
                // bf16 x bf16 products are exact in fp32, so fused or not the step rounds once.
                for (int i = 0; i < k; i++)
                    acc = fmaf(o_bf16_to_f32(w[((size_t)(i >> 1) * T + c) * 2 + (i & 1)]), o_bf16_to_f32(x->bf16[i]), acc);
            } else {
                size_t bb = tile_block_bytes(dtype);
                for (int b = 0; b < k / QB; b++) {
                    const uint8_t *blk = tile + b * bb;
                    int32_t dot = block_dot(dtype, blk, c, x->q8 + b * QB, x->sum[b]);
                    // acc += x.scale[b] * d[c] * (float)dot: the scale product rounds, then one fma.
                    float sd = x->scale[b] * tile_block_scale(dtype, blk, c);
                    acc = fmaf(sd, (float)dot, acc);
                }
            }
            y[t * T + c] = acc;
        }
    }
}

// reference src/ops.c:13-18. The sum of squares runs in index order. The compiler vectorises the
// squares 8 (then 4) at a time and adds them one by one, so those elements add a rounded square;
// the last n % 4 elements (after the 8- and 4-wide chunks) each take one fused multiply-add.
int o_rmsnorm_fused_from(int n) {
    int n8 = n & ~7, rem = n - n8;
    return rem >= 4 ? n8 + 4 : n8;
}

void o_rmsnorm(float *y, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    int split = o_rmsnorm_fused_from(n);
    for (int i = 0; i < split; i++) ss = ss + x[i] * x[i];
    for (int i = split; i < n; i++) ss = fmaf(x[i], x[i], ss);
    float s = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) y[i] = (x[i] * s) * w[i];
}

// reference src/ops.c:29-40 — adjacent pairs (2i, 2i+1), angle pos * theta^(-2i/hd).
void o_rope(float *v, int n_heads, int head_dim, int pos, float theta) {
    for (int i = 0; i < head_dim / 2; i++) {
        float angle = (float)pos * powf(theta, -2.0f * (float)i / (float)head_dim);
        float c = cosf(angle), s = sinf(angle);
        for (int h = 0; h < n_heads; h++) {
            float *p = v + h * head_dim + 2 * i;
            float a = p[0], b = p[1];
            p[0] = fmaf(a, c, -(b * s));
            p[1] = fmaf(a, s, b * c);
        }
    }
}

// reference src/ops.c:49-51
void o_silu_mul(float *h, const float *gate, int n) {
    for (int i = 0; i < n; i++) h[i] = h[i] * (gate[i] / (1.0f + o_expf(-gate[i])));
}

// reference src/ops.c:42-47, 58-73 — scores by a sequential sum of rounded products over head_dim,
// softmax with a sequential sum, then the value mix as one fma chain per output element over positions.
void o_attend(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int head_dim, int stride) {
    float s[pos + 1];
    float scale = 1.0f / sqrtf((float)head_dim);
    for (int t = 0; t <= pos; t++) {
        const uint16_t *kt = k + (size_t)t * stride;
        float dot = 0.0f;
        for (int i = 0; i < head_dim; i++) dot = dot + q[i] * o_bf16_to_f32(kt[i]);   // rounded product, then add
        s[t] = dot * scale;
    }
    float mx = s[0], sum = 0.0f;
    for (int t = 1; t <= pos; t++) if (s[t] > mx) mx = s[t];
    for (int t = 0; t <= pos; t++) { s[t] = o_expf(s[t] - mx); sum += s[t]; }
    for (int t = 0; t <= pos; t++) s[t] /= sum;
    for (int i = 0; i < head_dim; i++) out[i] = 0.0f;
    for (int t = 0; t <= pos; t++) {
        const uint16_t *vt = v + (size_t)t * stride;
        for (int i = 0; i < head_dim; i++) out[i] = fmaf(s[t], o_bf16_to_f32(vt[i]), out[i]);
    }
}
