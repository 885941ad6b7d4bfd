// CTA-wide building blocks of the exact decode path. Every function is called by all threads of
// the block with uniform arguments and ends with a barrier. Floating-point steps use the _rn
// intrinsics, which the compiler never fuses or reorders, in the order the reference's scalar
// path rounds (its compiled arithmetic is restated and pinned in the oracle; the same order is
// written here):
//   matvec, quantised:  acc = fma(RN(sx[b] * d[c]), (float)dot[b][c], acc) over blocks b in order,
//                       where dot is the exact integer block dot (any order);
//   matvec, bf16:       acc = fma(w_i, x_i, acc) over inputs in order (products are exact);
//   matvec, f32:        acc = acc + RN(w_i x_i) up to split(K), then fma — split(n) = n & ~7, plus 4
//                       more when n % 8 >= 4 (the reference compiler's 8- then 4-wide vector loop);
//   rmsnorm:            the same split for the sum of squares, then s = 1/sqrt(ss/n + eps), (x*s)*w;
//   attention:          scores by a sequential sum of rounded products; softmax with libm-exact
//                       expf and a sequential sum; the value mix as an fma chain over positions.
#pragma once
#include "device.cuh"

namespace l3m {

enum { DT_F32 = 0, DT_BF16 = 1, DT_Q8 = 2, DT_Q4 = 3, DT_MX = 4 };

__host__ __device__ inline int fused_from(int n) {
    int n8 = n & ~7;
    return (n - n8) >= 4 ? n8 + 4 : n8;
}

__host__ __device__ inline int block_bytes(int dtype) {      // per 16-output tile and 32 inputs
    return dtype == DT_Q8 ? 544 : dtype == DT_Q4 ? 288 : dtype == DT_MX ? 272 : 0;
}
__host__ __device__ inline size_t tile_bytes(int dtype, int k) {
    if (dtype == DT_F32) return (size_t)k * kTile * 4;
    if (dtype == DT_BF16) return (size_t)k * kTile * 2;
    return (size_t)(k / kQB) * block_bytes(dtype);
}

// A prepared activation in shared memory.
struct Prep {
    int8_t *q8;       // n, 16-byte aligned
    float *scale;     // n/32
    int32_t *sum;     // n/32
    float *xf;        // n: the values the f32/bf16 kernels multiply (bf16-rounded for bf16)
};

// ---- prepare (reference src/pack.c:101-122)
__device__ inline void prepare(int dtype, const float *x, int n, const Prep &p) {
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nth >> 5;
    if (dtype == DT_F32) {
        for (int i = tid; i < n; i += nth) p.xf[i] = x[i];
    } else if (dtype == DT_BF16) {
        for (int i = tid; i < n; i += nth) p.xf[i] = l3m_bf16_to_f32(l3m_f32_to_bf16(x[i]));
    } else {
        for (int b = warp; b < n / kQB; b += nw) {
            float v = x[b * kQB + lane];
            float a = fabsf(v);
            float amax = warp_max_f32(a > 0.0f ? a : 0.0f);          // a NaN never raises the maximum
            float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            int8_t q = (int8_t)__float2int_rn(__fmul_rn(v, inv));
            p.q8[b * kQB + lane] = q;
            int s = warp_sum_i32((int)q);
            if (lane == 0) {
                p.scale[b] = __fdiv_rn(amax, 127.0f);
                p.sum[b] = s;
            }
        }
    }
    __syncthreads();
}

// ---- quantised block dots. Tile layout per 32-input block (reference src/kernels.h:1-10):
// q8: d[16] f16 then q[8 groups][16 lanes][4] (value + 128); q4/mxfp4: scales then
// q[4 groups][16 lanes][4 bytes], byte j of a lane holding inputs 8g+j (low) and 8g+4+j (high).
// Each result is written as {RN(sx[b] * d[c]), (float)dot} for the fp32 chain.

// One q8 block of one tile by a whole warp: lane l loads 16 bytes = group l/4, outputs 4(l%4)..+3.
// Returns the exact integer dot of output *c (offset removed); lanes with bit 2 clear hold each
// output once.
__device__ __forceinline__ int q8_dot(uint4 w, int lane, uint32_t xw, int32_t xsum, int *c) {
    int p0 = dp4a_us(w.x, xw, 0), p1 = dp4a_us(w.y, xw, 0), p2 = dp4a_us(w.z, xw, 0), p3 = dp4a_us(w.w, xw, 0);
    const bool b4 = lane & 16, b3 = lane & 8;
    // Reduce the 8 groups (lane bits 4,3,2) while spreading the 4 outputs over those bits.
    int k0 = (b4 ? p2 : p0) + __shfl_xor_sync(0xffffffffu, b4 ? p0 : p2, 16);
    int k1 = (b4 ? p3 : p1) + __shfl_xor_sync(0xffffffffu, b4 ? p1 : p3, 16);
    int k = (b3 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    *c = 4 * (lane & 3) + (b4 ? 2 : 0) + (b3 ? 1 : 0);
    return k - 128 * xsum;
}

__device__ __forceinline__ void q8_block(uint4 w, const uint8_t *blk, int lane, uint32_t xw, int32_t xsum, float xscale, float2 *dst) {
    int c;
    const int dot = q8_dot(w, lane, xw, xsum, &c);
    if (!(lane & 4)) {
        float d = l3m_f16_to_f32(ld_nc_u16(blk + 2 * c));
        dst[c] = make_float2(__fmul_rn(xscale, d), __int2float_rn(dot));
    }
}

// The 16-entry mxfp4 table (doubled e2m1 + 16) applied to 4 nibble selectors in s[15:0].
__device__ __forceinline__ uint32_t mx_lut16(uint32_t s) {
    const uint32_t sm = s & 0x7777u;
    const uint32_t pos = prmt(0x13121110u, 0x1C181614u, sm);     // 16 17 18 19 20 22 24 28
    const uint32_t neg = prmt(0x0D0E0F10u, 0x04080A0Cu, sm);     // 16 15 14 13 12 10  8  4
    const uint32_t m = prmt(0x80808080u, 0x80808080u, s) ^ 0x80808080u;   // 0x7F where bit 3 is set
    return (pos & ~m) | (neg & m);
}

// One 4-bit block of one tile by a half warp: t = lane % 16 loads 16 bytes = group t/4, outputs
// 4(t%4)..+3. Returns the exact integer dot of output *c (offset removed); every t holds a distinct output.
template <bool MX>
__device__ __forceinline__ int q4_dot(uint4 w, int t, const uint32_t *xw, int32_t xsum, int *c) {
    const int g = t >> 2;
    const uint32_t xl = xw[2 * g], xh = xw[2 * g + 1];
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
    int p[4];
    if (MX) {
        const uint32_t xa = prmt(xl, xh, 0x5140u), xb = prmt(xl, xh, 0x7362u);   // inputs 0 4 1 5 and 2 6 3 7
#pragma unroll
        for (int j = 0; j < 4; j++) p[j] = dp4a_us(mx_lut16(ww[j]), xa, dp4a_us(mx_lut16(ww[j] >> 16), xb, 0));
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) p[j] = dp4a_us(ww[j] & 0x0F0F0F0Fu, xl, dp4a_us((ww[j] >> 4) & 0x0F0F0F0Fu, xh, 0));
    }
    const bool b3 = t & 8, b2 = t & 4;
    int k0 = (b3 ? p[2] : p[0]) + __shfl_xor_sync(0xffffffffu, b3 ? p[0] : p[2], 8);
    int k1 = (b3 ? p[3] : p[1]) + __shfl_xor_sync(0xffffffffu, b3 ? p[1] : p[3], 8);
    int k = (b2 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, b2 ? k0 : k1, 4);
    *c = 4 * (t & 3) + (b3 ? 2 : 0) + (b2 ? 1 : 0);
    return k - (MX ? 16 : 8) * xsum;
}

template <bool MX>
__device__ __forceinline__ void q4_block(uint4 w, const uint8_t *blk, int t, const uint32_t *xw, int32_t xsum, float xscale,
                                         float2 *dst, bool valid) {
    int c;
    const int dot = q4_dot<MX>(w, t, xw, xsum, &c);
    if (valid) {
        float d = MX ? l3m_e8m0_half(ld_nc_u8(blk + c)) : l3m_f16_to_f32(ld_nc_u16(blk + 2 * c));
        dst[c] = make_float2(__fmul_rn(xscale, d), __int2float_rn(dot));
    }
}

// Block dots of tiles [c0, c0 + ntl) into scratch[(tile * nb + b) * 16 + c]; four blocks in flight per warp.
__device__ inline void block_dots(int dtype, const uint8_t *tiles, int k, int c0, int ntl, const Prep &p, float2 *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nb = k / kQB, items = ntl * nb, bb = block_bytes(dtype);
    const size_t tb = (size_t)nb * bb;
    const uint32_t *xw = (const uint32_t *)p.q8;
    if (dtype == DT_Q8) {
        for (int base = warp; base < items; base += 4 * nw) {
            uint4 w[4];
            const uint8_t *blk[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                int it = base + u * nw;
                if (it < items) {
                    int ti = it / nb, b = it - ti * nb;
                    blk[u] = tiles + (size_t)(c0 + ti) * tb + (size_t)b * bb;
                    w[u] = ld_nc_v4(blk[u] + 32 + lane * 16);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                int it = base + u * nw;
                if (it < items) {
                    int ti = it / nb, b = it - ti * nb;
                    q8_block(w[u], blk[u], lane, xw[b * 8 + (lane >> 2)], p.sum[b], p.scale[b], scratch + ((size_t)ti * nb + b) * kTile);
                }
            }
        }
    } else {
        const int half = lane >> 4, t = lane & 15, sb = dtype == DT_MX ? 16 : 32;
        for (int base = 2 * warp; base < items; base += 8 * nw) {
            uint4 w[4];
            const uint8_t *blk[4];
            int bs[4], tis[4];
            bool ok[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                int it0 = base + 2 * u * nw;                  // both halves agree on whether to run
                int it = it0 + half;
                ok[u] = it < items;
                int itc = ok[u] ? it : (it0 < items ? it0 : 0);
                tis[u] = itc / nb;
                bs[u] = itc - tis[u] * nb;
                blk[u] = tiles + (size_t)(c0 + tis[u]) * tb + (size_t)bs[u] * bb;
                if (it0 < items) w[u] = ld_nc_v4(blk[u] + sb + t * 16);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (base + 2 * u * nw >= items) continue;     // uniform across the warp
                float2 *dst = scratch + ((size_t)tis[u] * nb + bs[u]) * kTile;
                if (dtype == DT_MX) q4_block<true>(w[u], blk[u], t, xw + bs[u] * 8, p.sum[bs[u]], p.scale[bs[u]], dst, ok[u]);
                else q4_block<false>(w[u], blk[u], t, xw + bs[u] * 8, p.sum[bs[u]], p.scale[bs[u]], dst, ok[u]);
            }
        }
    }
}

// y = tiles[t0, t1) . x for one CTA, exact. out(o, value) receives output o in [0, 16 (t1 - t0)).
// scratch holds scratch_pairs float2 (quantised dtypes; at least k/32 * 16).
template <class Out>
__device__ void matvec_exact(int dtype, const uint8_t *tiles, int k, int t0, int t1, const Prep &p, float2 *scratch,
                             int scratch_pairs, Out out) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (t1 <= t0) return;
    if (dtype == DT_F32 || dtype == DT_BF16) {
        const size_t tb = tile_bytes(dtype, k);
        const int n = (t1 - t0) * kTile, split = fused_from(k);
        for (int o = tid; o < n; o += nth) {
            const uint8_t *tile = tiles + (size_t)(t0 + (o >> 4)) * tb;
            const int c = o & 15;
            float acc = 0.0f;
            if (dtype == DT_BF16) {
                const uint32_t *w = (const uint32_t *)tile + c;
#pragma unroll 8
                for (int q = 0; q < k / 2; q++) {
                    uint32_t v = ld_nc_u32(w + (size_t)q * kTile);
                    acc = __fmaf_rn(l3m_bits_f32(v << 16), p.xf[2 * q], acc);
                    acc = __fmaf_rn(l3m_bits_f32(v & 0xFFFF0000u), p.xf[2 * q + 1], acc);
                }
            } else {
                const float *w = (const float *)tile + c;
#pragma unroll 8
                for (int i = 0; i < split; i++) acc = __fadd_rn(acc, __fmul_rn(__ldg(w + (size_t)i * kTile), p.xf[i]));
                for (int i = split; i < k; i++) acc = __fmaf_rn(__ldg(w + (size_t)i * kTile), p.xf[i], acc);
            }
            out(o, acc);
        }
        __syncthreads();
        return;
    }
    const int nb = k / kQB;
    int chunk = scratch_pairs / (nb * kTile);
    if (chunk < 1) chunk = 1;
    for (int c0 = t0; c0 < t1; c0 += chunk) {
        const int ntl = min(t1 - c0, chunk);
        block_dots(dtype, tiles, k, c0, ntl, p, scratch);
        __syncthreads();
        for (int o = tid; o < ntl * kTile; o += nth) {
            const float2 *s = scratch + (size_t)(o >> 4) * nb * kTile + (o & 15);
            float acc = 0.0f;
#pragma unroll 4
            for (int b = 0; b < nb; b++) {
                float2 v = s[(size_t)b * kTile];
                acc = __fmaf_rn(v.x, v.y, acc);
            }
            out((c0 - t0) * kTile + o, acc);
        }
        __syncthreads();
    }
}

// ---- rmsnorm (reference src/ops.c:13-18). tmp: n floats of shared scratch; red: one float.
__device__ inline void rmsnorm_exact(const float *x, const float *w, int n, float eps, float *y, float *tmp, float *red) {
    const int tid = threadIdx.x, nth = blockDim.x, split = fused_from(n);
    for (int i = tid; i < split; i += nth) tmp[i] = __fmul_rn(x[i], x[i]);
    __syncthreads();
    if (tid == 0) {
        float ss = 0.0f;
        const float4 *t4 = (const float4 *)tmp;
        for (int i = 0; i < split / 4; i++) {
            float4 v = t4[i];
            ss = __fadd_rn(ss, v.x); ss = __fadd_rn(ss, v.y); ss = __fadd_rn(ss, v.z); ss = __fadd_rn(ss, v.w);
        }
        for (int i = split; i < n; i++) ss = __fmaf_rn(x[i], x[i], ss);
        *red = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    }
    __syncthreads();
    const float s = *red;
    for (int i = tid; i < n; i += nth) y[i] = __fmul_rn(__fmul_rn(x[i], s), __ldg(w + i));
    __syncthreads();
}

// ---- RoPE on one head in place (reference src/ops.c:29-40): cs[i] = {cos, sin} of pair i at this position.
__device__ inline void rope_exact(float *v, int hd, const float2 *cs) {
    for (int i = threadIdx.x; i < hd / 2; i += blockDim.x) {
        const float2 c = cs[i];
        const float a = v[2 * i], b = v[2 * i + 1];
        v[2 * i] = __fmaf_rn(a, c.x, -__fmul_rn(b, c.y));
        v[2 * i + 1] = __fmaf_rn(a, c.y, __fmul_rn(b, c.x));
    }
    __syncthreads();
}

__device__ __forceinline__ float expf_libm(float x, const uint32_t *list, const uint32_t *index) {
    return l3m_expf_exact(x, list, index);
}

// ---- one head of attention at position pos (reference src/ops.c:42-47, 58-73). Rows 0..pos-1 of
// this head's K and V cache are in global memory, `stride` elements apart; row pos is kcur/vcur
// (16-byte aligned). scores: >= pos + 1 floats of shared scratch; red: >= 33 floats. hd % 8 == 0.
__device__ __forceinline__ uint4 ld_row8(const uint16_t *p, bool vec) {
    if (vec) return ld_cg_v4(p);
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; j++) h[j] = ld_cg_u16(p + j);
    return make_uint4(h[0] | (uint32_t)h[1] << 16, h[2] | (uint32_t)h[3] << 16, h[4] | (uint32_t)h[5] << 16, h[6] | (uint32_t)h[7] << 16);
}

__device__ inline void attend_exact(const float *q, const uint16_t *kc, const uint16_t *vc, int stride, const uint16_t *kcur,
                                    const uint16_t *vcur, int pos, int hd, float *scores, float *out, float *red,
                                    const uint32_t *elist, const uint32_t *eindex) {
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
    const bool vec = stride % 8 == 0 && ((uintptr_t)kc & 15) == 0;
    for (int t = tid; t <= pos; t += nth) {
        float dot = 0.0f;
        for (int i = 0; i < hd; i += 8) {
            uint4 v = t == pos ? *(const uint4 *)(kcur + i) : ld_row8(kc + (size_t)t * stride + i, vec);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                dot = __fadd_rn(dot, __fmul_rn(q[i + 2 * j], l3m_bits_f32(u[j] << 16)));
                dot = __fadd_rn(dot, __fmul_rn(q[i + 2 * j + 1], l3m_bits_f32(u[j] & 0xFFFF0000u)));
            }
        }
        scores[t] = __fmul_rn(dot, scale);
    }
    __syncthreads();
    // The reference takes the running maximum from scores[0] with a strict >: NaN scores after the
    // first are skipped, a NaN first score stays. The maximum of the rest is order-free.
    float m = -INFINITY;
    for (int t = tid; t <= pos; t += nth) m = fmaxf(m, scores[t]);
    m = warp_max_f32(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = -INFINITY;
        for (int w = 0; w < (nth >> 5); w++) mm = fmaxf(mm, red[w]);
        red[32] = scores[0] != scores[0] ? scores[0] : mm;
    }
    __syncthreads();
    const float mx = red[32];
    for (int t = tid; t <= pos; t += nth) scores[t] = expf_libm(__fsub_rn(scores[t], mx), elist, eindex);
    __syncthreads();
    if (tid == 0) {
        float sum = 0.0f;
        for (int t = 0; t <= pos; t++) sum = __fadd_rn(sum, scores[t]);
        red[32] = sum;
    }
    __syncthreads();
    const float sum = red[32];
    for (int t = tid; t <= pos; t += nth) scores[t] = __fdiv_rn(scores[t], sum);
    __syncthreads();
    for (int i = tid; i < hd; i += nth) {
        float acc = 0.0f;
#pragma unroll 8
        for (int t = 0; t < pos; t++) acc = __fmaf_rn(scores[t], l3m_bf16_to_f32(ld_cg_u16(vc + (size_t)t * stride + i)), acc);
        out[i] = __fmaf_rn(scores[pos], l3m_bf16_to_f32(vcur[i]), acc);
    }
    __syncthreads();
}

// SiLU gate (reference src/ops.c:49-51): h * (g / (1 + expf(-g))).
__device__ __forceinline__ float silu_mul(float h, float g, const uint32_t *elist, const uint32_t *eindex) {
    return __fmul_rn(h, __fdiv_rn(g, __fadd_rn(1.0f, expf_libm(-g, elist, eindex))));
}

}  // namespace l3m
