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
// Distance between consecutive tiles copied into shared memory. f32/bf16 tiles are copied one by
// one, 64 bytes apart beyond their size: the two half-warps of a warp (two tiles, one output each
// per lane) then read opposite halves of the banks.
__host__ __device__ inline size_t staged_stride(int dtype, int k) {
    return tile_bytes(dtype, k) + (dtype == DT_F32 || dtype == DT_BF16 ? 64 : 0);
}

// A prepared activation in shared memory.
struct Prep {
    int8_t *q8;       // n, 16-byte aligned
    float *scale;     // n/32
    int32_t *sum;     // n/32
    float *xf;        // n: the values the f32/bf16 kernels multiply (bf16-rounded for bf16)
};

// ---- prepare (reference src/pack.c:101-122)
// One quantisation step: the 8 lanes j = 0..7 of a warp's quarter hold the 4 values each of one
// 32-input block b (lanes with ok false hold zeros and store nothing); every lane of the warp calls.
__device__ __forceinline__ void quant_block4(const float4 v, int b, int j, bool ok, const Prep &p) {
    const float a0 = fabsf(v.x), a1 = fabsf(v.y), a2 = fabsf(v.z), a3 = fabsf(v.w);
    // a NaN never raises the maximum; the maximum of the rest is order-free
    float m = fmaxf(fmaxf(a0 > 0.0f ? a0 : 0.0f, a1 > 0.0f ? a1 : 0.0f), fmaxf(a2 > 0.0f ? a2 : 0.0f, a3 > 0.0f ? a3 : 0.0f));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    const float inv = m > 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
    const int q0 = (int8_t)__float2int_rn(__fmul_rn(v.x, inv)), q1 = (int8_t)__float2int_rn(__fmul_rn(v.y, inv));
    const int q2 = (int8_t)__float2int_rn(__fmul_rn(v.z, inv)), q3 = (int8_t)__float2int_rn(__fmul_rn(v.w, inv));
    int sm = q0 + q1 + q2 + q3;
    sm += __shfl_xor_sync(0xffffffffu, sm, 4);
    sm += __shfl_xor_sync(0xffffffffu, sm, 2);
    sm += __shfl_xor_sync(0xffffffffu, sm, 1);
    if (ok) {
        ((uint32_t *)(p.q8 + b * kQB))[j] = (uint32_t)(q0 & 0xFF) | (uint32_t)(q1 & 0xFF) << 8 | (uint32_t)(q2 & 0xFF) << 16 | (uint32_t)(q3 & 0xFF) << 24;
        if (j == 0) {
            p.scale[b] = __fdiv_rn(m, 127.0f);
            p.sum[b] = sm;
        }
    }
}

static __device__ __noinline__ void prepare(int dtype, const float *x, int n, const Prep p) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (dtype == DT_F32) {
#pragma unroll 1
        for (int i = tid; i < n; i += nth) p.xf[i] = x[i];
    } else if (dtype == DT_BF16) {
#pragma unroll 1
        for (int i = tid; i < n; i += nth) p.xf[i] = l3m_bf16_to_f32(l3m_f32_to_bf16(x[i]));
    } else {
        // 8 threads per 32-input block, 4 inputs each (x 16-byte aligned in shared memory); a warp takes
        // 4 blocks per step and every lane of it runs every step, so the shuffles always see the whole warp.
        const int j = tid & 7, sub = (tid & 31) >> 3, nblk = n / kQB;
#pragma unroll 1
        for (int b0 = (tid >> 5) * 4; b0 < nblk; b0 += (nth >> 5) * 4) {
            const int b = b0 + sub;
            const bool ok = b < nblk;
            const float4 v = ok ? ((const float4 *)(x + b * kQB))[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            quant_block4(v, b, j, ok, p);
        }
    }
    __syncthreads();
}

// Copy n floats global -> shared: asynchronous 16-byte copies when both sides allow (the caller
// commits, then waits with cp_async_wait_all + __syncthreads), else plain loads.
__device__ __forceinline__ void stage_f32(float *dst, const float *src, int n) {
    if ((n & 3) == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0) {
        #pragma unroll 1
        for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) cp_async16(dst + i, src + i);
    } else {
        #pragma unroll 1
        for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldg(src + i);
    }
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

// Four consecutive rows' block (rows 4r4..4r4+3 of a tile), loaded ahead of use: 16 bytes per group
// (q8: 8 groups, q4/mxfp4: 4) and the four scales.
struct QLoad4 { uint4 w[8]; uint2 d; };

// GEN: generic loads (the block may be in shared memory), else streaming global loads.
template <int DT, bool GEN>
__device__ __forceinline__ void qload4(QLoad4 &q, const uint8_t *blk, int r4) {
    if (DT == DT_Q8) {
        const uint8_t *g = blk + 32 + 16 * r4;
#pragma unroll
        for (int j = 0; j < 8; j++) q.w[j] = GEN ? *(const uint4 *)(g + 64 * j) : ld_stream_v4(g + 64 * j);
        q.d = GEN ? *(const uint2 *)(blk + 8 * r4) : ld_stream_v2(blk + 8 * r4);
    } else {
        const uint8_t *g = blk + (DT == DT_MX ? 16 : 32) + 16 * r4;
#pragma unroll
        for (int j = 0; j < 4; j++) q.w[j] = GEN ? *(const uint4 *)(g + 64 * j) : ld_stream_v4(g + 64 * j);
        if (DT == DT_MX) q.d = make_uint2(GEN ? *(const uint32_t *)(blk + 4 * r4) : ld_stream_u32(blk + 4 * r4), 0);
        else q.d = GEN ? *(const uint2 *)(blk + 8 * r4) : ld_stream_v2(blk + 8 * r4);
    }
}

__device__ __forceinline__ uint4 lds_u4_ord(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t lds_u32_ord(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint2 lds_u2_ord(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
    return v;
}
// qload4 from a block at shared-window address blk (shared-space loads, in program order).
template <int DT>
__device__ __forceinline__ void qload4_shared(QLoad4 &q, uint32_t blk, int r4) {
    if (DT == DT_Q8) {
        const uint32_t g = blk + 32 + 16 * r4;
#pragma unroll
        for (int j = 0; j < 8; j++) q.w[j] = lds_u4_ord(g + 64 * j);
        q.d = lds_u2_ord(blk + 8 * r4);
    } else {
        const uint32_t g = blk + (DT == DT_MX ? 16 : 32) + 16 * r4;
#pragma unroll
        for (int j = 0; j < 4; j++) q.w[j] = lds_u4_ord(g + 64 * j);
        if (DT == DT_MX) q.d = make_uint2(lds_u32_ord(blk + 4 * r4), 0);
        else q.d = lds_u2_ord(blk + 8 * r4);
    }
}

__device__ __forceinline__ uint32_t u4_at(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// Exact integer dot of row c (0..3) of a QLoad4 with the block's prepared activation words xw[0..7],
// offset removed (the reference's acc_i - offset * sum, src/kernels_scalar.c:37-43, 57-71).
template <int DT>
__device__ __forceinline__ int qdot4(const QLoad4 &q, int c, const uint32_t *xw, int32_t xsum) {
    int s = 0, t = 0;
    if (DT == DT_Q8) {
#pragma unroll
        for (int j = 0; j < 8; j += 2) { s = dp4a_us(u4_at(q.w[j], c), xw[j], s); t = dp4a_us(u4_at(q.w[j + 1], c), xw[j + 1], t); }
        return s + t - 128 * xsum;
    } else if (DT == DT_Q4) {
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const uint32_t w = u4_at(q.w[g], c);
            s = dp4a_us(w & 0x0F0F0F0Fu, xw[2 * g], s);
            t = dp4a_us((w >> 4) & 0x0F0F0F0Fu, xw[2 * g + 1], t);
        }
        return s + t - 8 * xsum;
    } else {
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const uint32_t w = u4_at(q.w[g], c), xl = xw[2 * g], xh = xw[2 * g + 1];
            // bytes 0,1 of the word select inputs 0 4 1 5 of the group; bytes 2,3 select 2 6 3 7
            s = dp4a_us(mx_lut16(w), prmt(xl, xh, 0x5140u), s);
            t = dp4a_us(mx_lut16(w >> 16), prmt(xl, xh, 0x7362u), t);
        }
        return s + t - 16 * xsum;
    }
}

template <int DT>
__device__ __forceinline__ float qscale4(const uint2 &d, int c) {
    if (DT == DT_MX) return l3m_e8m0_half((uint8_t)(d.x >> (8 * c)));
    const uint32_t w = c < 2 ? d.x : d.y;
    return l3m_f16_to_f32((uint16_t)(c & 1 ? w >> 16 : w));
}

// Single-row forms (one output's block), used where one thread owns one (output, block) item.
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

template <int DT>
__device__ __forceinline__ int qdot(const QLoad &q, const uint32_t *xw, int32_t xsum) {
    QLoad4 q4;
#pragma unroll
    for (int j = 0; j < 8; j++) q4.w[j] = make_uint4(q.w[j], 0, 0, 0);
    q4.d = make_uint2(q.d, 0);
    return qdot4<DT>(q4, 0, xw, xsum);
}

template <int DT>
__device__ __forceinline__ float qscale(uint32_t d) { return DT == DT_MX ? l3m_e8m0_half((uint8_t)d) : l3m_f16_to_f32((uint16_t)d); }

// Outputs [0, n_out) of the tiles at `tiles` (n_out a multiple of 16), exact. The (4 outputs, block)
// items of a chunk of outputs are dealt to threads output-fastest, kQU items in flight per thread;
// each output's {RN(sx[b] * d), (float)dot} goes to scratch[b * m + o]. Then one thread per output
// runs the fp32 chain in block order.
constexpr int kQU = 2;
// Tiles [0, ntA) come from `tiles`, tiles from ntA on from tilesB. GEN: generic loads (tiles may be
// a copy in shared memory), else streaming global loads.
template <int DT, bool GEN>
__device__ void qmatvec(const uint8_t *tiles, const uint8_t *tilesB, int ntA, int k, int n_out, const Prep &p, float2 *scratch,
                        int scratch_pairs, float *y) {
    const int tid = threadIdx.x, nth = blockDim.x, nb = k / kQB, bb = block_bytes(DT);
    const size_t tb = (size_t)nb * bb;
    const uint32_t *xw = (const uint32_t *)p.q8;
    int chunk = (scratch_pairs / nb) & ~(kTile - 1);           // >= 16: callers size scratch for one tile
    if (chunk > n_out) chunk = n_out;
    for (int o0 = 0; o0 < n_out; o0 += chunk) {
        const int m = min(chunk, n_out - o0), m4 = m >> 2, items = m4 * nb, t0 = o0 >> 4;
        // item i = b * m4 + quad; this thread starts at i = tid and steps by nth
        int b = tid / m4, qd = tid - b * m4;
        const int db = nth / m4, dq = nth - db * m4;
        #pragma unroll 1
        for (int i = tid; i < items; i += kQU * nth) {
            QLoad4 q[kQU];
            int bs[kQU], qs[kQU];
#pragma unroll
            for (int u = 0; u < kQU; u++) {
                bs[u] = b; qs[u] = qd;
                if (i + u * nth < items) {
                    const int ti = t0 + (qd >> 2);
                    const uint8_t *tile = ti < ntA ? tiles + (size_t)ti * tb : tilesB + (size_t)(ti - ntA) * tb;
                    qload4<DT, GEN>(q[u], tile + (size_t)b * bb, qd & 3);
                }
                qd += dq; b += db;
                if (qd >= m4) { qd -= m4; b++; }
            }
#pragma unroll
            for (int u = 0; u < kQU; u++) {
                if (i + u * nth < items) {
                    const uint4 x0 = *(const uint4 *)(xw + 8 * bs[u]), x1 = *(const uint4 *)(xw + 8 * bs[u] + 4);
                    const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    const float sx = p.scale[bs[u]];
                    const int32_t xs = p.sum[bs[u]];
                    float4 r0, r1;
                    r0.x = __fmul_rn(sx, qscale4<DT>(q[u].d, 0)); r0.y = __int2float_rn(qdot4<DT>(q[u], 0, xv, xs));
                    r0.z = __fmul_rn(sx, qscale4<DT>(q[u].d, 1)); r0.w = __int2float_rn(qdot4<DT>(q[u], 1, xv, xs));
                    r1.x = __fmul_rn(sx, qscale4<DT>(q[u].d, 2)); r1.y = __int2float_rn(qdot4<DT>(q[u], 2, xv, xs));
                    r1.z = __fmul_rn(sx, qscale4<DT>(q[u].d, 3)); r1.w = __int2float_rn(qdot4<DT>(q[u], 3, xv, xs));
                    float4 *dst = (float4 *)(scratch + (size_t)bs[u] * m + 4 * qs[u]);
                    dst[0] = r0;
                    dst[1] = r1;
                }
            }
        }
        __syncthreads();
        #pragma unroll 1
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

// Shared-memory loads by shared-window address (the chains below), in program order with every other
// memory access and barrier (volatile, memory clobber): the loops that use them already issue each
// load where it must go, so the compiler has nothing to reorder, and it must not move one above the
// barrier or store that makes its data ready. Arithmetic still schedules freely around them.
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) { return __uint_as_float(lds_u32(a)); }
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a) : "memory");
    return v;
}

// One output's bf16 chain over a tile staged in shared memory (the reference's order, products exact
// inside each fma): word q of the output at wa + 64 q holds inputs 2q (low half) and 2q + 1; x (fp32)
// at xa. 32 inputs per iteration in two halves, one half's loads in flight while the other computes.
__device__ __forceinline__ void ld8w(uint32_t (&w)[8], float4 (&x)[4], uint32_t wa, uint32_t xa, int q) {
#pragma unroll
    for (int j = 0; j < 8; j++) w[j] = lds_u32(wa + 64 * (q + j));
#pragma unroll
    for (int j = 0; j < 4; j++) x[j] = lds_f4(xa + 8 * q + 16 * j);
}
__device__ __forceinline__ float fma8w(float acc, const uint32_t (&w)[8], const float4 (&x)[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        acc = __fmaf_rn(l3m_bits_f32(w[2 * j] << 16), x[j].x, acc);
        acc = __fmaf_rn(l3m_bits_f32(w[2 * j] & 0xFFFF0000u), x[j].y, acc);
        acc = __fmaf_rn(l3m_bits_f32(w[2 * j + 1] << 16), x[j].z, acc);
        acc = __fmaf_rn(l3m_bits_f32(w[2 * j + 1] & 0xFFFF0000u), x[j].w, acc);
    }
    return acc;
}
__device__ __forceinline__ float chain_bf16_shared(uint32_t wa, uint32_t xa, int k) {
    const int nw = k >> 1, n16 = nw & ~15;
    float acc = 0.0f;
    int q = 0;
    if (n16) {
        uint32_t wA[8], wB[8];
        float4 xA[4], xB[4];
        ld8w(wA, xA, wa, xa, 0);
#pragma unroll 1
        for (; q < n16; q += 16) {
            ld8w(wB, xB, wa, xa, q + 8);
            acc = fma8w(acc, wA, xA);
            const int qn = q + 16 < n16 ? q + 16 : q;
            ld8w(wA, xA, wa, xa, qn);
            acc = fma8w(acc, wB, xB);
        }
    }
#pragma unroll 1
    for (; q < nw; q++) {
        const uint32_t v = lds_u32(wa + 64 * q);
        acc = __fmaf_rn(l3m_bits_f32(v << 16), lds_f32(xa + 8 * q), acc);
        acc = __fmaf_rn(l3m_bits_f32(v & 0xFFFF0000u), lds_f32(xa + 8 * q + 4), acc);
    }
    return acc;
}

// The same for an f32 tile (input i of the output at wa + 64 i): rounded products added up to
// split, fmas after (the reference build's chain); 16 inputs per iteration in two halves.
__device__ __forceinline__ void ld8f(float (&w)[8], float4 (&x)[2], uint32_t wa, uint32_t xa, int i) {
#pragma unroll
    for (int j = 0; j < 8; j++) w[j] = lds_f32(wa + 64 * (i + j));
    x[0] = lds_f4(xa + 4 * i);
    x[1] = lds_f4(xa + 4 * i + 16);
}
__device__ __forceinline__ float add8f(float acc, const float (&w)[8], const float4 (&x)[2]) {
    const float xv[8] = {x[0].x, x[0].y, x[0].z, x[0].w, x[1].x, x[1].y, x[1].z, x[1].w};
#pragma unroll
    for (int j = 0; j < 8; j++) acc = __fadd_rn(acc, __fmul_rn(w[j], xv[j]));
    return acc;
}
__device__ __forceinline__ float chain_f32_shared(uint32_t wa, uint32_t xa, int k, int split) {
    float acc = 0.0f;
    int i = 0;
    const int s16 = split & ~15;
    if (s16) {
        float wA[8], wB[8];
        float4 xA[2], xB[2];
        ld8f(wA, xA, wa, xa, 0);
#pragma unroll 1
        for (; i < s16; i += 16) {
            ld8f(wB, xB, wa, xa, i + 8);
            acc = add8f(acc, wA, xA);
            const int in = i + 16 < s16 ? i + 16 : i;
            ld8f(wA, xA, wa, xa, in);
            acc = add8f(acc, wB, xB);
        }
    }
#pragma unroll 1
    for (; i < split; i++) acc = __fadd_rn(acc, __fmul_rn(lds_f32(wa + 64 * i), lds_f32(xa + 4 * i)));
#pragma unroll 1
    for (; i < k; i++) acc = __fmaf_rn(lds_f32(wa + 64 * i), lds_f32(xa + 4 * i), acc);
    return acc;
}

// One out-of-line copy per quantised dtype (a layer runs only its own dtype's code).
template <int DT>
static __device__ __noinline__ void qmatvec_call(const uint8_t *tiles, const uint8_t *tilesB, int ntA, int k, int n_out, const Prep p,
                                                 float2 *scratch, int scratch_pairs, float *y) {
    qmatvec<DT, true>(tiles, tilesB, ntA, k, n_out, p, scratch, scratch_pairs, y);
}

// f32 / bf16 tiles ([K][16] f32, [K/2][16][2] bf16) [0, n/16) at base (the first ns staged), one
// output per thread.
template <int DT>
static __device__ __noinline__ void matvec_wide(const uint8_t *base, int k, int n, const Prep p, float *y, const uint8_t *staged, int ns) {
    const int tid = threadIdx.x, nth = blockDim.x;
    // f32 / bf16 (tiles [K][16] f32, [K/2][16][2] bf16): one thread per output walks its row in input
    // order, the reference's chain; lanes 0-15 and 16-31 of a warp take two tiles.
    const int split = fused_from(k);
    const size_t sst = staged_stride(DT, k), tb = tile_bytes(DT, k);
    const uint32_t xa = (uint32_t)__cvta_generic_to_shared(p.xf);
#pragma unroll 1
    for (int o = tid; o < n; o += nth) {
        const int t = o >> 4, c = o & 15;
        if (t < ns) {
            const uint32_t wa = (uint32_t)__cvta_generic_to_shared(staged + (size_t)t * sst) + 4 * c;
            y[o] = DT == DT_BF16 ? chain_bf16_shared(wa, xa, k) : chain_f32_shared(wa, xa, k, split);
            continue;
        }
        const uint8_t *tile = base + (size_t)t * tb;
        float acc = 0.0f;
        if (DT == DT_BF16) {
            const uint32_t *w = (const uint32_t *)tile + c;
            int q = 0;
#pragma unroll 1
            for (; q + 8 <= k / 2; q += 8) {
                uint32_t v[8];
#pragma unroll
                for (int j = 0; j < 8; j++) v[j] = ld_stream_u32(w + (size_t)(q + j) * kTile);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    acc = __fmaf_rn(l3m_bits_f32(v[j] << 16), p.xf[2 * (q + j)], acc);
                    acc = __fmaf_rn(l3m_bits_f32(v[j] & 0xFFFF0000u), p.xf[2 * (q + j) + 1], acc);
                }
            }
#pragma unroll 1
            for (; q < k / 2; q++) {
                const uint32_t v = ld_stream_u32(w + (size_t)q * kTile);
                acc = __fmaf_rn(l3m_bits_f32(v << 16), p.xf[2 * q], acc);
                acc = __fmaf_rn(l3m_bits_f32(v & 0xFFFF0000u), p.xf[2 * q + 1], acc);
            }
        } else {
            const float *w = (const float *)tile + c;
#pragma unroll 8
            for (int i = 0; i < split; i++) acc = __fadd_rn(acc, __fmul_rn(__ldg(w + (size_t)i * kTile), p.xf[i]));
#pragma unroll 1
            for (int i = split; i < k; i++) acc = __fmaf_rn(__ldg(w + (size_t)i * kTile), p.xf[i], acc);
        }
        y[o] = acc;
    }
    __syncthreads();
}

// y = tiles[t0, t1) . x for one CTA, exact: y[o] for o in [0, 16 (t1 - t0)) (shared memory).
// scratch holds scratch_pairs float2 (quantised dtypes; at least k/32). staged, ns: a copy of tiles
// [t0, t0 + ns) in shared memory, staged_stride(dtype, k) bytes apart, read instead of global memory.
static __device__ __noinline__ void matvec_exact(int dtype, const uint8_t *tiles, int k, int t0, int t1, const Prep p, float2 *scratch,
                                                 int scratch_pairs, float *y, const uint8_t *staged = nullptr, int ns = 0) {
    if (t1 <= t0) return;
    const size_t tb = tile_bytes(dtype, k);
    const uint8_t *base = tiles + (size_t)t0 * tb;
    const int n = (t1 - t0) * kTile;
    const uint8_t *ta = ns > 0 ? staged : base, *tbb = ns > 0 ? base + (size_t)ns * tb : base;
    const int nta = ns > 0 ? ns : 1 << 30;
    if (dtype == DT_Q8) { qmatvec_call<DT_Q8>(ta, tbb, nta, k, n, p, scratch, scratch_pairs, y); return; }
    if (dtype == DT_Q4) { qmatvec_call<DT_Q4>(ta, tbb, nta, k, n, p, scratch, scratch_pairs, y); return; }
    if (dtype == DT_MX) { qmatvec_call<DT_MX>(ta, tbb, nta, k, n, p, scratch, scratch_pairs, y); return; }
    if (dtype == DT_BF16) matvec_wide<DT_BF16>(base, k, n, p, y, staged, ns);
    else matvec_wide<DT_F32>(base, k, n, p, y, staged, ns);
}

template <bool SQ>
static __device__ __noinline__ float seq_sum(const float *v, int n);

// ---- rmsnorm (reference src/ops.c:13-18). x 16-byte aligned, w in shared or global memory; red: one
// float. The sum of squares is the reference's sequential chain, run by thread 0. ps (when ps.kc is
// set): threads 32.. start attention's K/V copies
// meanwhile (attend_prestage), so that they land while the chain runs.
struct PreStage {
    const uint16_t *kc, *vc;
    int kstride, vstride, pos, hd;
    uint16_t *kvbuf, *vtbuf;
    int chunk;
};
template <bool VT>
__device__ __noinline__ void attend_prestage(const uint16_t *kc, const uint16_t *vc, int kstride, int vstride, int pos, int hd,
                                             uint16_t *kvbuf, uint16_t *vtbuf, int chunk, int tid = -1, int nth = 0);
__device__ __forceinline__ void side_prestage(const PreStage &ps) {
    if (ps.kc && threadIdx.x >= 32)
        attend_prestage<true>(ps.kc, ps.vc, ps.kstride, ps.vstride, ps.pos, ps.hd, ps.kvbuf, ps.vtbuf, ps.chunk, threadIdx.x - 32, blockDim.x - 32);
}
// The normalised vector's epilogue: y[i] = f(i) for i < n, and when pdt >= 0 the activation that a
// matrix of dtype pdt multiplies (prepare's output, from the same y values) in the same pass. f(i)
// is computed from 4 consecutive elements at a time when n is a multiple of 32 (quantised: 8 lanes per
// block, as prepare), else one element at a time.
template <class F>
__device__ __forceinline__ void norm_out(int n, float *y, int pdt, const Prep &p, const F &f) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (pdt >= DT_Q8 && n % kQB == 0) {
        const int j = tid & 7, sub = (tid & 31) >> 3, nblk = n / kQB;
#pragma unroll 1
        for (int b0 = (tid >> 5) * 4; b0 < nblk; b0 += (nth >> 5) * 4) {
            const int b = b0 + sub;
            const bool ok = b < nblk;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (ok) {
                const int i = b * kQB + 4 * j;
                v = make_float4(f(i), f(i + 1), f(i + 2), f(i + 3));
                *(float4 *)(y + i) = v;
            }
            quant_block4(v, b, j, ok, p);
        }
    } else {
#pragma unroll 1
        for (int i = tid; i < n; i += nth) {
            const float v = f(i);
            y[i] = v;
            if (pdt == DT_F32) p.xf[i] = v;
            else if (pdt == DT_BF16) p.xf[i] = l3m_bf16_to_f32(l3m_f32_to_bf16(v));
        }
    }
}

// pdt, p: also prepare the output for a matrix of dtype pdt (-1: do not).
static __device__ __noinline__ void rmsnorm_exact(const float *x, const float *w, int n, float eps, float *y, float *red, const PreStage ps = PreStage{},
                                                  int pdt = -1, const Prep p = Prep{}) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        const int split = fused_from(n);
        float ss = seq_sum<true>(x, split);
#pragma unroll 1
        for (int i = split; i < n; i++) ss = __fmaf_rn(x[i], x[i], ss);
        *red = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    } else {
        side_prestage(ps);
    }
    __syncthreads();
    const float sc = *red;
    norm_out(n, y, pdt, p, [&](int i) { return __fmul_rn(__fmul_rn(x[i], sc), w[i]); });
    __syncthreads();
}

// The variance chain of LayerNorm (reference src/ops.c:24 as built): d = x[i] - mean; the squares
// rounded on their own up to split (the vectorised part of the reference build), fused after.
__device__ __forceinline__ float chain_var(const float *v, float mean, int n, int split) {
    float acc = 0.0f;
    int i = 0;
    const float4 *v4 = (const float4 *)v;
    const int nf = split & ~3;
#pragma unroll 1
    for (; i < nf; i += 4) {
        const float4 r = v4[i >> 2];
        const float e[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int h = 0; h < 4; h++) {
            const float d = __fsub_rn(e[h], mean);
            acc = __fadd_rn(acc, __fmul_rn(d, d));
        }
    }
#pragma unroll 1
    for (; i < split; i++) { const float d = __fsub_rn(v[i], mean); acc = __fadd_rn(acc, __fmul_rn(d, d)); }
#pragma unroll 1
    for (; i < n; i++) { const float d = __fsub_rn(v[i], mean); acc = __fmaf_rn(d, d, acc); }
    return acc;
}

// LayerNorm (reference src/ops.c:20-27): sequential mean, the variance chain above, s = 1/sqrt(var/n
// + eps), y = fma((x - mean) * s, w, b). Thread 0 runs the chains; ps as in rmsnorm_exact.
static __device__ __noinline__ void layernorm_exact(const float *x, const float *w, const float *b, int n, float eps, float *y, float *red,
                                                    const PreStage ps = PreStage{}, int pdt = -1, const Prep p = Prep{}) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        const float mean = __fdiv_rn(seq_sum<false>(x, n), (float)n);
        const float var = chain_var(x, mean, n, fused_from(n));
        red[0] = mean;
        red[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var, (float)n), eps)));
    } else {
        side_prestage(ps);
    }
    __syncthreads();
    const float mean = red[0], sc = red[1];
    norm_out(n, y, pdt, p, [&](int i) { return __fmaf_rn(__fmul_rn(__fsub_rn(x[i], mean), sc), w[i], b[i]); });
    __syncthreads();
}

// GELU, tanh form (reference src/ops.c:53-56 as built: x + 0.044715 x^3 is one fma). tanhf is the
// device's: within a few ulp of the host libm's (which follows fdlibm's expm1f-based formulation),
// so GELU outputs, unlike every other step, are not bit-identical to the reference's.
__device__ __forceinline__ float gelu_tanh(float v) {
    const float inner = __fmaf_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v, v);
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(__fmul_rn(0.7978845608f, inner))));
}

// ---- RoPE on one head in place (reference src/ops.c:29-40): cs[i] = {cos, sin} of pair i at this position.
__device__ inline void rope_exact(float *v, int hd, const float2 *cs) {
    #pragma unroll 1
    for (int i = threadIdx.x; i < hd / 2; i += blockDim.x) {
        const float2 c = cs[i];
        const float a = v[2 * i], b = v[2 * i + 1];
        v[2 * i] = __fmaf_rn(a, c.x, -__fmul_rn(b, c.y));
        v[2 * i + 1] = __fmaf_rn(a, c.y, __fmul_rn(b, c.x));
    }
    __syncthreads();
}

// One out-of-line copy for every caller (attention's softmax, the SiLU gate): code size matters more
// than a call here.
static __device__ __noinline__ float expf_libm(float x, const uint32_t *tab) {
    return l3m_expf_exact(x, tab);
}

// ---- one head of attention at position pos (reference src/ops.c:42-47, 58-73).
// K rows 0..pos-1 are in global memory, kstride elements apart; row pos is kcur (shared, 16-byte
// aligned). V: with VT false, rows like K (vstride apart), row pos in vcur; with VT true, the cache
// is transposed — element i of position t at vc[i * vstride + t], vstride >= pos + 1 rounded up to
// 8 — and element i of row pos is vcur[i]. scores: >= pos + 1 floats of shared scratch (16-byte aligned); red: >= 33 floats.
// kvbuf: chunk * (hd + 8) bf16 of staging; vtbuf (VT only): hd * attn_vt_stride(chunk) bf16.
// hd % 8 == 0; chunk a multiple of 8. prestaged: attend_prestage has run for this call.
__device__ __forceinline__ uint4 ld_row8(const uint16_t *p, bool vec) {
    if (vec) return ld_cg_v4(p);
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; j++) h[j] = ld_cg_u16(p + j);
    return make_uint4(h[0] | (uint32_t)h[1] << 16, h[2] | (uint32_t)h[3] << 16, h[4] | (uint32_t)h[5] << 16, h[6] | (uint32_t)h[7] << 16);
}

// Row stride (elements) of the transposed V staging buffer: 4 x odd words, so the 16-byte reads of 8
// consecutive rows fall in distinct bank groups.
__host__ __device__ constexpr int attn_vt_stride(int chunk) { return ((chunk + 15) & ~15) + 8; }

// Start the copies of everything attention at pos reads that exists before row pos: K rows
// [0, min(chunk, pos)) and, with VT, V positions [0, min(chunk, pos + 1)) (position pos itself is
// patched later). Needs nothing of this position, so it can run before q, k and v are known. Run
// by threads tid of nth (every thread of the CTA by default, or a subset); each thread waits for its
// own copies (cp_async_wait_all) before the barrier that precedes reading them.
template <bool VT>
__device__ __noinline__ void attend_prestage(const uint16_t *kc, const uint16_t *vc, int kstride, int vstride, int pos, int hd,
                                             uint16_t *kvbuf, uint16_t *vtbuf, int chunk, int tid, int nth) {
    if (tid < 0) { tid = threadIdx.x; nth = blockDim.x; }
    const int rs = hd + 8, h8 = hd / 8, vs = attn_vt_stride(chunk);
    const bool kvec = kstride % 8 == 0 && ((uintptr_t)kc & 15) == 0;
    const bool vvec = vstride % 8 == 0 && ((uintptr_t)vc & 15) == 0;
    const int nk = min(chunk, pos);
    {
        const int dr = nth / h8, dj = nth - dr * h8;
        int r = tid / h8, j = tid - r * h8;
        #pragma unroll 1
        for (int e = tid; e < nk * h8; e += nth) {
            uint16_t *dst = kvbuf + r * rs + j * 8;
            const uint16_t *src = kc + (size_t)r * kstride + j * 8;
            if (kvec) cp_async16(dst, src);
            else *(uint4 *)dst = ld_row8(src, false);
            j += dj; r += dr;
            if (j >= h8) { j -= h8; r++; }
        }
    }
    if (VT) {
        const int p8 = (min(chunk, pos + 1) + 7) >> 3, di = nth / p8, dp = nth - di * p8;
        int i = tid / p8, pc = tid - i * p8;
        #pragma unroll 1
        for (int e = tid; e < hd * p8; e += nth) {
            uint16_t *dst = vtbuf + i * vs + pc * 8;
            const uint16_t *src = vc + (size_t)i * vstride + pc * 8;
            if (vvec) cp_async16(dst, src);
            else *(uint4 *)dst = ld_row8(src, false);
            pc += dp; i += di;
            if (pc >= p8) { pc -= p8; i++; }
        }
    }
    cp_async_commit();
}

// K rows [c0, c0 + cnt) into kvbuf (row r at r * (hd + 8)); row pos from kcur. Asynchronous where
// aligned (the caller commits, waits and synchronises).
static __device__ __noinline__ void stage_k_rows(uint16_t *kvbuf, const uint16_t *kc, int kstride, const uint16_t *kcur, int pos, int hd, int c0, int cnt,
                                          bool kvec) {
    const int tid = threadIdx.x, nth = blockDim.x, rs = hd + 8, h8 = hd / 8;
#pragma unroll 1
    for (int e = tid; e < cnt * h8; e += nth) {
        const int r = e / h8, i = (e - r * h8) * 8, t = c0 + r;
        uint16_t *dst = kvbuf + r * rs + i;
        if (t == pos) *(uint4 *)dst = *(const uint4 *)(kcur + i);
        else if (kvec) cp_async16(dst, kc + (size_t)t * kstride + i);
        else *(uint4 *)dst = ld_row8(kc + (size_t)t * kstride + i, false);
    }
    cp_async_commit();
}

// V of positions [c0, c0 + cnt) into shared memory. VT: vtbuf[i * vs + r], one 8-position piece per
// copy (positions past pos in a piece are never read; position pos itself is patched from vcur by
// the thread that reads its column, after the copies have landed). Else rows into kvbuf as K.
template <bool VT>
__device__ __noinline__ void stage_v_rows(uint16_t *kvbuf, uint16_t *vtbuf, const uint16_t *vc, int vstride, const uint16_t *vcur, int pos, int hd,
                                          int c0, int cnt, int chunk, bool vvec) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (VT) {
        const int p8 = (cnt + 7) >> 3, vs = attn_vt_stride(chunk);
#pragma unroll 1
        for (int e = tid; e < hd * p8; e += nth) {
            const int i = e / p8, pc = e - i * p8;
            uint16_t *dst = vtbuf + i * vs + pc * 8;
            const uint16_t *src = vc + (size_t)i * vstride + c0 + pc * 8;
            if (vvec) cp_async16(dst, src);
            else *(uint4 *)dst = ld_row8(src, false);
        }
    } else {
        stage_k_rows(kvbuf, vc, vstride, vcur, pos, hd, c0, cnt, vvec);
        return;
    }
    cp_async_commit();
}

// Sequential fp32 sum of v[0..n) (v in shared memory, 16-byte aligned) in index order, by the
// calling thread; each term squared first (rounded) with SQ. 64 values per iteration in two halves:
// one half's loads are in flight while the other half's 32 dependent adds run (about 150 cycles,
// enough to cover a shared-memory load while bulk copies land in the same memory), and no register
// copies between steps.
template <bool SQ>
__device__ __forceinline__ float add32(float acc, const float4 (&r)[8]) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float e[4] = {r[j].x, r[j].y, r[j].z, r[j].w};
#pragma unroll
        for (int h = 0; h < 4; h++) acc = __fadd_rn(acc, SQ ? __fmul_rn(e[h], e[h]) : e[h]);
    }
    return acc;
}
template <bool SQ>
static __device__ __noinline__ float seq_sum(const float *v, int n) {
    const uint32_t va = (uint32_t)__cvta_generic_to_shared(v);
    const int n64 = n & ~63;
    float acc = 0.0f;
    int i = 0;
    if (n64) {
        float4 a[8], b[8];
#pragma unroll
        for (int j = 0; j < 8; j++) a[j] = lds_f4(va + 16 * j);
#pragma unroll 1
        for (; i < n64; i += 64) {
#pragma unroll
            for (int j = 0; j < 8; j++) b[j] = lds_f4(va + 4 * i + 128 + 16 * j);
            acc = add32<SQ>(acc, a);
            const int in = i + 64 < n64 ? i + 64 : i;
#pragma unroll
            for (int j = 0; j < 8; j++) a[j] = lds_f4(va + 4 * in + 16 * j);
            acc = add32<SQ>(acc, b);
        }
    }
#pragma unroll 1
    for (; i + 4 <= n; i += 4) {
        const float4 t = lds_f4(va + 4 * i);
        acc = __fadd_rn(acc, SQ ? __fmul_rn(t.x, t.x) : t.x);
        acc = __fadd_rn(acc, SQ ? __fmul_rn(t.y, t.y) : t.y);
        acc = __fadd_rn(acc, SQ ? __fmul_rn(t.z, t.z) : t.z);
        acc = __fadd_rn(acc, SQ ? __fmul_rn(t.w, t.w) : t.w);
    }
#pragma unroll 1
    for (; i < n; i++) {
        const float t = lds_f32(va + 4 * i);
        acc = __fadd_rn(acc, SQ ? __fmul_rn(t, t) : t);
    }
    return acc;
}

// Attention's two chains, 32 steps per iteration in two halves (one half's loads in flight while the
// other's 16 dependent steps run). A score: the sequential sum of rounded products q[i] * k[i] (k
// bf16, 8 per 16 bytes); row, q in shared memory, 16-byte aligned; hd a multiple of 8.
__device__ __forceinline__ float dot8(float dot, const uint4 kv, const float4 q0, const float4 q1) {
    dot = __fadd_rn(dot, __fmul_rn(q0.x, l3m_bits_f32(kv.x << 16)));
    dot = __fadd_rn(dot, __fmul_rn(q0.y, l3m_bits_f32(kv.x & 0xFFFF0000u)));
    dot = __fadd_rn(dot, __fmul_rn(q0.z, l3m_bits_f32(kv.y << 16)));
    dot = __fadd_rn(dot, __fmul_rn(q0.w, l3m_bits_f32(kv.y & 0xFFFF0000u)));
    dot = __fadd_rn(dot, __fmul_rn(q1.x, l3m_bits_f32(kv.z << 16)));
    dot = __fadd_rn(dot, __fmul_rn(q1.y, l3m_bits_f32(kv.z & 0xFFFF0000u)));
    dot = __fadd_rn(dot, __fmul_rn(q1.z, l3m_bits_f32(kv.w << 16)));
    dot = __fadd_rn(dot, __fmul_rn(q1.w, l3m_bits_f32(kv.w & 0xFFFF0000u)));
    return dot;
}
__device__ __forceinline__ uint4 lds_u4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
    return v;
}
// 16 steps' operands: two 16-byte pieces of the bf16 vector at ra (+16) and four float4 at fa.
struct Ops16 {
    uint4 k0, k1;
    float4 f0, f1, f2, f3;
};
__device__ __forceinline__ void ld16(Ops16 &o, uint32_t ra, uint32_t fa) {
    o.k0 = lds_u4(ra);
    o.k1 = lds_u4(ra + 16);
    o.f0 = lds_f4(fa);
    o.f1 = lds_f4(fa + 16);
    o.f2 = lds_f4(fa + 32);
    o.f3 = lds_f4(fa + 48);
}
__device__ __forceinline__ float score_dot(const uint16_t *row, const float *q, int hd) {
    const uint32_t ra = (uint32_t)__cvta_generic_to_shared(row), qa = (uint32_t)__cvta_generic_to_shared(q);
    float dot = 0.0f;
    int i = 0;
    const int h32 = hd & ~31;
    if (h32) {
        Ops16 A, B;
        ld16(A, ra, qa);
#pragma unroll 1
        for (; i < h32; i += 32) {
            ld16(B, ra + 2 * (i + 16), qa + 4 * (i + 16));
            dot = dot8(dot, A.k0, A.f0, A.f1);
            dot = dot8(dot, A.k1, A.f2, A.f3);
            const int in = i + 32 < h32 ? i + 32 : i;
            ld16(A, ra + 2 * in, qa + 4 * in);
            dot = dot8(dot, B.k0, B.f0, B.f1);
            dot = dot8(dot, B.k1, B.f2, B.f3);
        }
    }
#pragma unroll 1
    for (; i < hd; i += 8) dot = dot8(dot, lds_u4(ra + 2 * i), lds_f4(qa + 4 * i), lds_f4(qa + 4 * i + 16));
    return dot;
}
// The value mix of one output element: acc = fma(p[r], v[r], acc) over positions in order, v a
// transposed column (bf16, 8 positions per 16 bytes); col and p in shared memory, 16-byte aligned.
__device__ __forceinline__ float vmix8(float acc, const uint4 v, const float4 p0, const float4 p1) {
    acc = __fmaf_rn(p0.x, l3m_bits_f32(v.x << 16), acc); acc = __fmaf_rn(p0.y, l3m_bits_f32(v.x & 0xFFFF0000u), acc);
    acc = __fmaf_rn(p0.z, l3m_bits_f32(v.y << 16), acc); acc = __fmaf_rn(p0.w, l3m_bits_f32(v.y & 0xFFFF0000u), acc);
    acc = __fmaf_rn(p1.x, l3m_bits_f32(v.z << 16), acc); acc = __fmaf_rn(p1.y, l3m_bits_f32(v.z & 0xFFFF0000u), acc);
    acc = __fmaf_rn(p1.z, l3m_bits_f32(v.w << 16), acc); acc = __fmaf_rn(p1.w, l3m_bits_f32(v.w & 0xFFFF0000u), acc);
    return acc;
}
__device__ __forceinline__ float vmix_col(const uint16_t *col, const float *pp, int cnt, float acc) {
    const uint32_t ca = (uint32_t)__cvta_generic_to_shared(col), pa = (uint32_t)__cvta_generic_to_shared(pp);
    int r = 0;
    const int c32 = cnt & ~31;
    if (c32) {
        Ops16 A, B;
        ld16(A, ca, pa);
#pragma unroll 1
        for (; r < c32; r += 32) {
            ld16(B, ca + 2 * (r + 16), pa + 4 * (r + 16));
            acc = vmix8(acc, A.k0, A.f0, A.f1);
            acc = vmix8(acc, A.k1, A.f2, A.f3);
            const int rn = r + 32 < c32 ? r + 32 : r;
            ld16(A, ca + 2 * rn, pa + 4 * rn);
            acc = vmix8(acc, B.k0, B.f0, B.f1);
            acc = vmix8(acc, B.k1, B.f2, B.f3);
        }
    }
#pragma unroll 1
    for (; r + 8 <= cnt; r += 8) acc = vmix8(acc, lds_u4(ca + 2 * r), lds_f4(pa + 4 * r), lds_f4(pa + 4 * r + 16));
#pragma unroll 1
    for (; r < cnt; r++) acc = __fmaf_rn(lds_f32(pa + 4 * r), l3m_bits_f32(lds_u32(ca + 2 * (r & ~1)) << (r & 1 ? 0 : 16) & 0xFFFF0000u), acc);
    return acc;
}

template <bool VT>
__device__ __noinline__ void attend_exact(const float *q, const uint16_t *kc, const uint16_t *vc, int kstride, int vstride, const uint16_t *kcur,
                             const uint16_t *vcur, int pos, int hd, float *scores, float *out, float *red, const uint32_t *etab,
                             uint16_t *kvbuf, uint16_t *vtbuf, int chunk, bool prestaged) {
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
    const bool kvec = kstride % 8 == 0 && ((uintptr_t)kc & 15) == 0;
    const bool vvec = vstride % 8 == 0 && ((uintptr_t)vc & 15) == 0;
    const int n = pos + 1, rs = hd + 8, vs = attn_vt_stride(chunk);
    if (!prestaged) attend_prestage<VT>(kc, vc, kstride, vstride, pos, hd, kvbuf, vtbuf, chunk);
    // Scores: one thread per row, from K rows staged in shared memory (coalesced copies); each dot is
    // the sequential sum of rounded products, 8 inputs per step with the next step's loads in flight.
    float m = -INFINITY;
#pragma unroll 1
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int cnt = min(chunk, n - c0);
        if (c0 > 0) {
            __syncthreads();
            stage_k_rows(kvbuf, kc, kstride, kcur, pos, hd, c0, cnt, kvec);
        } else if (pos < cnt) {                              // the first chunk's rows < pos are prestaged
#pragma unroll 1
            for (int i = tid * 8; i < hd; i += nth * 8) *(uint4 *)(kvbuf + pos * rs + i) = *(const uint4 *)(kcur + i);
        }
        cp_async_wait_all();
        __syncthreads();
#pragma unroll 1
        for (int r = tid; r < cnt; r += nth) {
            const float dot = score_dot(kvbuf + r * rs, q, hd);
            const float sc = __fmul_rn(dot, scale);
            scores[c0 + r] = sc;
            m = fmaxf(m, sc);
        }
    }
    __syncthreads();
    if (!VT) stage_v_rows<VT>(kvbuf, vtbuf, vc, vstride, vcur, pos, hd, 0, min(chunk, n), chunk, vvec);   // reuses the K buffer
    // The reference takes the running maximum from scores[0] with a strict >: NaN scores after the
    // first are skipped (fmaxf drops them), a NaN first score stays. The maximum of the rest is order-free.
    m = warp_max_f32(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float mx = -INFINITY;                                    // warp count a multiple of 4 (red 16-byte aligned)
#pragma unroll 1
    for (int w = 0; w < (nth >> 5); w += 4) {
        const float4 r = *(const float4 *)(red + w);
        mx = fmaxf(mx, fmaxf(fmaxf(r.x, r.y), fmaxf(r.z, r.w)));
    }
    if (scores[0] != scores[0]) mx = scores[0];
#pragma unroll 1
    for (int t = tid; t < n; t += nth) scores[t] = expf_libm(__fsub_rn(scores[t], mx), etab);
    __syncthreads();
    if (tid == 0) red[32] = seq_sum<false>(scores, n);      // the sequential sum
    __syncthreads();
    const float sum = red[32];
#pragma unroll 1
    for (int t = tid; t < n; t += nth) scores[t] = __fdiv_rn(scores[t], sum);
    cp_async_wait_all();
    __syncthreads();
    float acc = 0.0f;                                        // thread i < hd: output element i
#pragma unroll 1
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int cnt = min(chunk, n - c0);
        if (c0 > 0) {
            __syncthreads();
            stage_v_rows<VT>(kvbuf, vtbuf, vc, vstride, vcur, pos, hd, c0, cnt, chunk, vvec);
            cp_async_wait_all();
            __syncthreads();
        }
        if (tid < hd) {
            const float *pp = scores + c0;                   // c0 is a multiple of 8
            int r = 0;
            if (VT) {
                uint16_t *col = vtbuf + tid * vs;
                if (pos - c0 < cnt) col[pos - c0] = vcur[tid];
                acc = vmix_col(col, pp, cnt, acc);
            } else {
                const uint16_t *col = kvbuf + tid;
#pragma unroll 1
                for (; r < cnt; r++) acc = __fmaf_rn(pp[r], l3m_bf16_to_f32(col[r * rs]), acc);
            }
        }
    }
#pragma unroll 1
    for (int i = tid; i < hd; i += nth) out[i] = acc;
    __syncthreads();
}

// SiLU gate (reference src/ops.c:49-51): h * (g / (1 + expf(-g))).
__device__ __forceinline__ float silu_mul(float h, float g, const uint32_t *etab) {
    return __fmul_rn(h, __fdiv_rn(g, __fadd_rn(1.0f, expf_libm(-g, etab))));
}

}  // namespace l3m
