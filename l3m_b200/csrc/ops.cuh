// CTA-wide building blocks of the exact decode path. Every function is called by all threads of
// the block with uniform arguments and ends with a barrier. Floating-point steps use the _rn
// intrinsics, which the compiler never fuses or reorders, in the order the reference's scalar
// path rounds (its compiled arithmetic is restated and pinned in the oracle; the same order is
// written here):
//   matvec, quantised:  acc = fma(RN(sx[b] * d[c]), (float)dot[b][c], acc) over blocks b in order,
//                       where dot is the exact integer block dot (computed by any thread);
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
static __device__ __noinline__ void prepare(int dtype, const float *x, int n, const Prep p) {
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
//   q8:    d[16] f16, then q[8 groups][16 rows][4] u8 (value + 128): group g holds inputs 4g..4g+3
//   q4:    d[16] f16, then q[4 groups][16 rows][4] bytes: byte j of group g holds inputs 8g+j (low
//          nibble) and 8g+4+j (high nibble)
//   mxfp4: e[16] e8m0, then codes as q4
// One row's block is 8 (q8) or 4 (q4, mxfp4) words 64 bytes apart, so one thread computes a whole
// exact block dot with dp4a and no cross-lane traffic, and the 16 rows of a tile read one 64-byte
// run per group.

// The 16-entry mxfp4 table (doubled e2m1 + 16) applied to 4 nibble selectors in s[15:0].
__device__ __forceinline__ uint32_t mx_lut16(uint32_t s) {
    const uint32_t sm = s & 0x7777u;
    const uint32_t pos = prmt(0x13121110u, 0x1C181614u, sm);     // 16 17 18 19 20 22 24 28
    const uint32_t neg = prmt(0x0D0E0F10u, 0x04080A0Cu, sm);     // 16 15 14 13 12 10  8  4
    const uint32_t m = prmt(0x80808080u, 0x80808080u, s) ^ 0x80808080u;   // 0x7F where bit 3 is set
    return (pos & ~m) | (neg & m);
}

// One row's block, loaded ahead of use: its words and its scale bits.
struct QLoad { uint32_t w[8]; uint32_t d; };

template <int DT>
__device__ __forceinline__ void qload(QLoad &q, const uint8_t *blk, int c) {
    if (DT == DT_Q8) {
        const uint32_t *g = (const uint32_t *)(blk + 32) + c;
#pragma unroll
        for (int j = 0; j < 8; j++) q.w[j] = __ldg(g + 16 * j);
        q.d = ld_nc_u16(blk + 2 * c);
    } else if (DT == DT_Q4) {
        const uint32_t *g = (const uint32_t *)(blk + 32) + c;
#pragma unroll
        for (int j = 0; j < 4; j++) q.w[j] = __ldg(g + 16 * j);
        q.d = ld_nc_u16(blk + 2 * c);
    } else {
        const uint32_t *g = (const uint32_t *)(blk + 16) + c;
#pragma unroll
        for (int j = 0; j < 4; j++) q.w[j] = __ldg(g + 16 * j);
        q.d = ld_nc_u8(blk + c);
    }
}

// Exact integer dot of a loaded block with the block's 8 prepared activation words xw[0..7], offset
// removed (the reference's acc_i - offset * sum, src/kernels_scalar.c:37-43, 57-71).
template <int DT>
__device__ __forceinline__ int qdot(const QLoad &q, const uint32_t *xw, int32_t xsum) {
    int s = 0, t = 0;
    if (DT == DT_Q8) {
#pragma unroll
        for (int j = 0; j < 8; j += 2) { s = dp4a_us(q.w[j], xw[j], s); t = dp4a_us(q.w[j + 1], xw[j + 1], t); }
        return s + t - 128 * xsum;
    } else if (DT == DT_Q4) {
#pragma unroll
        for (int g = 0; g < 4; g++) {
            s = dp4a_us(q.w[g] & 0x0F0F0F0Fu, xw[2 * g], s);
            t = dp4a_us((q.w[g] >> 4) & 0x0F0F0F0Fu, xw[2 * g + 1], t);
        }
        return s + t - 8 * xsum;
    } else {
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const uint32_t xl = xw[2 * g], xh = xw[2 * g + 1];
            // bytes 0,1 of the word select inputs 0 4 1 5 of the group; bytes 2,3 select 2 6 3 7
            s = dp4a_us(mx_lut16(q.w[g]), prmt(xl, xh, 0x5140u), s);
            t = dp4a_us(mx_lut16(q.w[g] >> 16), prmt(xl, xh, 0x7362u), t);
        }
        return s + t - 16 * xsum;
    }
}

template <int DT>
__device__ __forceinline__ float qscale(uint32_t d) { return DT == DT_MX ? l3m_e8m0_half((uint8_t)d) : l3m_f16_to_f32((uint16_t)d); }

// Outputs [0, n_out) of the tiles at `tiles`, exact. The (output, block) items of a chunk of outputs
// are dealt to threads output-fastest, kQU blocks in flight per thread; each stores {RN(sx[b] * d),
// (float)dot} at scratch[b * m + o]. Then one thread per output runs the fp32 chain in block order.
constexpr int kQU = 4;
template <int DT>
__device__ void qmatvec(const uint8_t *tiles, int k, int n_out, const Prep &p, float2 *scratch, int scratch_pairs, float *y) {
    const int tid = threadIdx.x, nth = blockDim.x, nb = k / kQB, bb = block_bytes(DT);
    const size_t tb = (size_t)nb * bb;
    const uint32_t *xw = (const uint32_t *)p.q8;
    int chunk = scratch_pairs / nb;
    if (chunk > n_out) chunk = n_out;
    for (int o0 = 0; o0 < n_out; o0 += chunk) {
        const int m = min(chunk, n_out - o0), items = m * nb;
        // item i = b * m + o; this thread starts at i = tid and steps by nth
        int b = tid / m, o = tid - b * m;
        const int db = nth / m, dor = nth - db * m;
        const uint8_t *base = tiles + (size_t)o0 / kTile * tb;   // o0 is a multiple of 16 unless chunk is not
        const int oc = o0 % kTile;
        for (int i = tid; i < items; i += kQU * nth) {
            QLoad q[kQU];
            int bs[kQU], os[kQU];
#pragma unroll
            for (int u = 0; u < kQU; u++) {
                bs[u] = b; os[u] = o;
                if (i + u * nth < items) {
                    const int oo = o + oc;
                    qload<DT>(q[u], base + (size_t)(oo >> 4) * tb + (size_t)b * bb, oo & 15);
                }
                o += dor; b += db;
                if (o >= m) { o -= m; b++; }
            }
#pragma unroll
            for (int u = 0; u < kQU; u++) {
                if (i + u * nth < items) {
                    const int dot = qdot<DT>(q[u], xw + 8 * bs[u], p.sum[bs[u]]);
                    scratch[(size_t)bs[u] * m + os[u]] = make_float2(__fmul_rn(p.scale[bs[u]], qscale<DT>(q[u].d)), __int2float_rn(dot));
                }
            }
        }
        __syncthreads();
        for (int oo = tid; oo < m; oo += nth) {
            const float2 *r = scratch + oo;
            float acc = 0.0f;
#pragma unroll 6
            for (int bb2 = 0; bb2 < nb; bb2++) {
                const float2 v = r[(size_t)bb2 * m];
                acc = __fmaf_rn(v.x, v.y, acc);
            }
            y[o0 + oo] = acc;
        }
        __syncthreads();
    }
}

// y = tiles[t0, t1) . x for one CTA, exact: y[o] for o in [0, 16 (t1 - t0)) (shared memory).
// scratch holds scratch_pairs float2 (quantised dtypes; at least k/32).
static __device__ __noinline__ void matvec_exact(int dtype, const uint8_t *tiles, int k, int t0, int t1, const Prep p, float2 *scratch,
                                                 int scratch_pairs, float *y) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (t1 <= t0) return;
    const size_t tb = tile_bytes(dtype, k);
    const uint8_t *base = tiles + (size_t)t0 * tb;
    const int n = (t1 - t0) * kTile;
    if (dtype == DT_Q8) { qmatvec<DT_Q8>(base, k, n, p, scratch, scratch_pairs, y); return; }
    if (dtype == DT_Q4) { qmatvec<DT_Q4>(base, k, n, p, scratch, scratch_pairs, y); return; }
    if (dtype == DT_MX) { qmatvec<DT_MX>(base, k, n, p, scratch, scratch_pairs, y); return; }
    // f32 / bf16 (tiles [K][16] f32, [K/2][16][2] bf16): one thread per output walks its row in input
    // order, the reference's chain.
    const int split = fused_from(k);
    for (int o = tid; o < n; o += nth) {
        const uint8_t *tile = base + (size_t)(o >> 4) * tb;
        const int c = o & 15;
        float acc = 0.0f;
        if (dtype == DT_BF16) {
            const uint32_t *w = (const uint32_t *)tile + c;
            int q = 0;
            for (; q + 8 <= k / 2; q += 8) {
                uint32_t v[8];
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] = __ldg(w + (size_t)(q + j) * kTile);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    acc = __fmaf_rn(l3m_bits_f32(v[j] << 16), p.xf[2 * (q + j)], acc);
                    acc = __fmaf_rn(l3m_bits_f32(v[j] & 0xFFFF0000u), p.xf[2 * (q + j) + 1], acc);
                }
            }
            for (; q < k / 2; q++) {
                const uint32_t v = __ldg(w + (size_t)q * kTile);
                acc = __fmaf_rn(l3m_bits_f32(v << 16), p.xf[2 * q], acc);
                acc = __fmaf_rn(l3m_bits_f32(v & 0xFFFF0000u), p.xf[2 * q + 1], acc);
            }
        } else {
            const float *w = (const float *)tile + c;
#pragma unroll 8
            for (int i = 0; i < split; i++) acc = __fadd_rn(acc, __fmul_rn(__ldg(w + (size_t)i * kTile), p.xf[i]));
            for (int i = split; i < k; i++) acc = __fmaf_rn(__ldg(w + (size_t)i * kTile), p.xf[i], acc);
        }
        y[o] = acc;
    }
    __syncthreads();
}

// ---- rmsnorm (reference src/ops.c:13-18). tmp: n floats of shared scratch; red: one float.
static __device__ __noinline__ void rmsnorm_exact(const float *x, const float *w, int n, float eps, float *y, float *tmp, float *red) {
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

static __device__ __noinline__ void attend_exact(const float *q, const uint16_t *kc, const uint16_t *vc, int stride, const uint16_t *kcur,
                                    const uint16_t *vcur, int pos, int hd, float *scores, float *out, float *red,
                                    const uint32_t *elist, const uint32_t *eindex, uint16_t *kvbuf, int chunk) {
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
    const bool vec = stride % 8 == 0 && ((uintptr_t)kc & 15) == 0 && ((uintptr_t)vc & 15) == 0;
    const int rs = hd + 8;                                   // padded row stride in the staging buffer (elements)
    // Rows 0..pos-1 come through shared memory in chunks: coalesced 16-byte loads, then each thread
    // walks its own row (scores) or its own column (value mix) out of the staging buffer.
    for (int c0 = 0; c0 <= pos; c0 += chunk) {
        const int n = min(chunk, pos + 1 - c0);
#pragma unroll 4
        for (int e = tid; e < n * (hd / 8); e += nth) {
            const int r = e / (hd / 8), i = (e - r * (hd / 8)) * 8, t = c0 + r;
            const uint4 v = t == pos ? *(const uint4 *)(kcur + i) : ld_row8(kc + (size_t)t * stride + i, vec);
            *(uint4 *)(kvbuf + r * rs + i) = v;
        }
        __syncthreads();
        for (int r = tid; r < n; r += nth) {
            const uint16_t *row = kvbuf + r * rs;
            float dot = 0.0f;
            for (int i = 0; i < hd; i += 8) {
                const uint4 v = *(const uint4 *)(row + i);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    dot = __fadd_rn(dot, __fmul_rn(q[i + 2 * j], l3m_bits_f32(u[j] << 16)));
                    dot = __fadd_rn(dot, __fmul_rn(q[i + 2 * j + 1], l3m_bits_f32(u[j] & 0xFFFF0000u)));
                }
            }
            scores[c0 + r] = __fmul_rn(dot, scale);
        }
        __syncthreads();
    }
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
    float acc = 0.0f;                                        // thread i < hd: output element i
    for (int c0 = 0; c0 <= pos; c0 += chunk) {
        const int n = min(chunk, pos + 1 - c0);
#pragma unroll 4
        for (int e = tid; e < n * (hd / 8); e += nth) {
            const int r = e / (hd / 8), i = (e - r * (hd / 8)) * 8, t = c0 + r;
            const uint4 v = t == pos ? *(const uint4 *)(vcur + i) : ld_row8(vc + (size_t)t * stride + i, vec);
            *(uint4 *)(kvbuf + r * rs + i) = v;
        }
        __syncthreads();
        if (tid < hd) {
#pragma unroll 8
            for (int r = 0; r < n; r++) acc = __fmaf_rn(scores[c0 + r], l3m_bf16_to_f32(kvbuf[r * rs + tid]), acc);
        }
        __syncthreads();
    }
    for (int i = tid; i < hd; i += nth) out[i] = acc;
    __syncthreads();
}

// SiLU gate (reference src/ops.c:49-51): h * (g / (1 + expf(-g))).
__device__ __forceinline__ float silu_mul(float h, float g, const uint32_t *elist, const uint32_t *eindex) {
    return __fmul_rn(h, __fdiv_rn(g, __fadd_rn(1.0f, expf_libm(-g, elist, eindex))));
}

}  // namespace l3m
