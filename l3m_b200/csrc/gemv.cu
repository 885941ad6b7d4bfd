// Standalone matvec kernels behind include/l3m_kernels.h: y = tiles . x on the device, with the
// reference's tile layout (src/kernels.h:1-10) and its scalar table's results (src/kernels_scalar.c).
//
// Exact table, quantised dtypes: every CTA takes a contiguous run of tiles; each thread computes the
// exact integer dots of 4 outputs x one 32-input block with dp4a from 16-byte loads (two such items
// in flight), then one thread per output runs the fp32 epilogue over the blocks in order.
// Exact table, f32/bf16: one thread per output runs the sequential chain over K (the order the
// reference rounds in). Fast table, f32/bf16: the chain is split over K across a warp and reduced
// with shuffles (reassociated, like the reference's AVX tables; tolerance-checked).
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include <mutex>
#include "ops.cuh"
#include "../../include/l3m_kernels.h"

using namespace l3m;

namespace {

thread_local char g_err[256];

int fail(cudaError_t e, const char *what) {
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return -1;
}
int fail_msg(const char *msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return -1;
}

constexpr int kThreads = 512;
constexpr int kScratchPairs = 4096;                 // 32 KB of block results per chunk
constexpr int kAttnChunk = 128;                     // KV rows staged in shared memory at a time

struct VecArg { const float *f32; const uint16_t *bf16; const int8_t *q8; const float *scale; const int32_t *sum; };

__host__ __device__ size_t prep_smem(int k) {                            // q8[k], scale[k/32], sum[k/32], xf[k], 16-byte aligned parts
    size_t a = ((size_t)k + 15) & ~(size_t)15, s = (((size_t)(k / 32 + 1)) * 4 + 15) & ~(size_t)15;
    return a + 2 * s + (size_t)k * 4;
}

__device__ Prep carve_prep(unsigned char *base, int k) {
    Prep p;
    size_t a = ((size_t)k + 15) & ~(size_t)15, s = (((size_t)(k / 32 + 1)) * 4 + 15) & ~(size_t)15;
    p.q8 = (int8_t *)base;
    p.scale = (float *)(base + a);
    p.sum = (int32_t *)(base + a + s);
    p.xf = (float *)(base + a + 2 * s);
    return p;
}

// Copy a prepared vector from global memory into the CTA's shared memory.
__device__ void load_prep(int dtype, const VecArg &x, int k, const Prep &p) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (dtype == DT_F32) for (int i = tid; i < k; i += nth) p.xf[i] = x.f32[i];
    else if (dtype == DT_BF16) for (int i = tid; i < k; i += nth) p.xf[i] = l3m_bf16_to_f32(x.bf16[i]);
    else {
        for (int i = tid; i < k; i += nth) p.q8[i] = x.q8[i];
        for (int i = tid; i < k / 32; i += nth) { p.scale[i] = x.scale[i]; p.sum[i] = x.sum[i]; }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads) gemv_exact_kernel(int dtype, float *y, const uint8_t *tiles, int ntiles, int k, VecArg x) {
    extern __shared__ __align__(16) unsigned char smem[];
    Prep p = carve_prep(smem, k);
    float2 *scratch = (float2 *)(smem + prep_smem(k));
    load_prep(dtype, x, k, p);
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x), t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    float *ys = (float *)(scratch + kScratchPairs);                    // this CTA's outputs, then to global
    matvec_exact(dtype, tiles, k, t0, t1, p, scratch, kScratchPairs, ys);
    for (int o = threadIdx.x; o < (t1 - t0) * kTile; o += blockDim.x) y[(size_t)t0 * kTile + o] = ys[o];
}

// Fast f32/bf16: one warp per tile; each half warp walks alternate 16-input chunks for its 16 outputs.
__global__ void __launch_bounds__(kThreads) gemv_fast_kernel(int dtype, float *y, const uint8_t *tiles, int ntiles, int k, VecArg x) {
    const int lane = threadIdx.x & 31, warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5), c = lane & 15, half = lane >> 4;
    const size_t tb = tile_bytes(dtype, k);
    for (int t = warp; t < ntiles; t += nwarps) {
        const uint8_t *tile = tiles + (size_t)t * tb;
        float a0 = 0.0f, a1 = 0.0f;
        if (dtype == DT_BF16) {
            const uint32_t *w = (const uint32_t *)tile + c;
            for (int q = half; q < k / 2; q += 2) {
                const uint32_t v = ld_nc_u32(w + (size_t)q * kTile);
                a0 = fmaf(l3m_bits_f32(v << 16), l3m_bf16_to_f32(x.bf16[2 * q]), a0);
                a1 = fmaf(l3m_bits_f32(v & 0xFFFF0000u), l3m_bf16_to_f32(x.bf16[2 * q + 1]), a1);
            }
        } else {
            const float *w = (const float *)tile + c;
            for (int i = half; i < k; i += 2) a0 = fmaf(__ldg(w + (size_t)i * kTile), x.f32[i], a0);
        }
        float acc = a0 + a1;
        acc += __shfl_xor_sync(0xffffffffu, acc, 16);
        if (!half) y[(size_t)t * kTile + c] = acc;
    }
}

// Exact integer block dots, one warp (q8) or half warp (q4, mxfp4) per (tile, block).
template <int DT>
__device__ void block_dots_items(int32_t *dots, const uint8_t *tiles, int ntiles, int k, const VecArg &x) {
    const int nb = k / kQB, bb = block_bytes(DT);
    const size_t tb = (size_t)nb * bb;
    const long long n = (long long)ntiles * kTile, items = n * nb;
    const uint32_t *xw = (const uint32_t *)x.q8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / n);
        const long long o = i - (long long)b * n;
        QLoad q;
        qload<DT>(q, tiles + (size_t)(o >> 4) * tb + (size_t)b * bb, (int)(o & 15));
        dots[o * nb + b] = qdot<DT>(q, xw + 8 * b, x.sum[b]);
    }
}

// Exact integer block dots: one thread per (output, block).
__global__ void block_dots_kernel(int dtype, int32_t *dots, const uint8_t *tiles, int ntiles, int k, VecArg x) {
    if (dtype == DT_Q8) block_dots_items<DT_Q8>(dots, tiles, ntiles, k, x);
    else if (dtype == DT_Q4) block_dots_items<DT_Q4>(dots, tiles, ntiles, k, x);
    else block_dots_items<DT_MX>(dots, tiles, ntiles, k, x);
}

// Unpack: one thread per (output, block).
__global__ void unpack_kernel(int dtype, int8_t *q, float *d, const uint8_t *tiles, int ntiles, int k) {
    const int nb = k / kQB, bb = block_bytes(dtype);
    const size_t tb = (size_t)nb * bb;
    const long long n = (long long)ntiles * kTile * nb;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < n; id += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(id % nb);
        const long long o = id / nb;
        const int t = (int)(o / kTile), c = (int)(o % kTile);
        const uint8_t *blk = tiles + (size_t)t * tb + (size_t)b * bb;
        int8_t *qo = q + o * k + b * kQB;
        if (dtype == DT_Q8) {
            d[o * nb + b] = l3m_f16_to_f32(ld_nc_u16(blk + 2 * c));
            for (int i = 0; i < kQB; i++) qo[i] = (int8_t)(ld_nc_u8(blk + 32 + ((i / 4) * kTile + c) * 4 + i % 4) - 128);
        } else {
            const int sb = dtype == DT_MX ? 16 : 32;
            d[o * nb + b] = dtype == DT_MX ? l3m_e8m0_half(ld_nc_u8(blk + c)) : l3m_f16_to_f32(ld_nc_u16(blk + 2 * c));
            for (int i = 0; i < kQB; i++) {
                const int g = i / 8, j = i % 8;
                const uint8_t byte = ld_nc_u8(blk + sb + (g * kTile + c) * 4 + (j & 3));
                const int nib = j < 4 ? (byte & 15) : (byte >> 4);
                qo[i] = (int8_t)(dtype == DT_MX ? l3m_mxfp4_value(nib) : nib - 8);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) prepare_kernel(int dtype, const float *x, int n, int8_t *q8, float *scale, int32_t *sum, uint16_t *bf16) {
    const int tid = threadIdx.x + blockIdx.x * blockDim.x, nth = blockDim.x * gridDim.x;
    if (dtype == DT_BF16) {
        for (int i = tid; i < n; i += nth) bf16[i] = l3m_f32_to_bf16(x[i]);
        return;
    }
    const int lane = threadIdx.x & 31, gw = tid >> 5, nw = nth >> 5;
    for (int b = gw; b < n / kQB; b += nw) {
        const float v = x[b * kQB + lane], a = fabsf(v);
        const float amax = warp_max_f32(a > 0.0f ? a : 0.0f);
        const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int8_t q = (int8_t)__float2int_rn(__fmul_rn(v, inv));
        q8[b * kQB + lane] = q;
        const int s = warp_sum_i32((int)q);
        if (lane == 0) { scale[b] = __fdiv_rn(amax, 127.0f); sum[b] = s; }
    }
}

__global__ void __launch_bounds__(kThreads) attend_kernel(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int hd,
                                                          int stride, const uint32_t *elist, const uint32_t *eindex) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *qs = (float *)smem, *o = qs + hd, *red = o + hd, *scores = red + 64;
    uint16_t *kcur = (uint16_t *)(scores + ((pos + 4) & ~3)), *vcur = kcur + hd, *kvbuf = vcur + hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        qs[i] = q[i];
        kcur[i] = k[(size_t)pos * stride + i];
        vcur[i] = v[(size_t)pos * stride + i];
    }
    __syncthreads();
    attend_exact<false>(qs, k, v, stride, stride, kcur, vcur, pos, hd, scores, o, red, elist, eindex, kvbuf, nullptr, kAttnChunk, false);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) out[i] = o[i];
}

VecArg vec_arg(const l3m_vec *x) { return VecArg{x->f32, x->bf16, x->q8, x->scale, x->sum}; }

int grid_for(int ntiles) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    int g = 2 * sms;
    return ntiles < g ? (ntiles > 0 ? ntiles : 1) : g;
}

}  // namespace

// ---- expf exception list on the device (shared with the decode engine)
#include "expf_exceptions.inc"

extern "C" int l3m_expf_tables(const uint32_t **list, const uint32_t **index) {
    static std::mutex mu;
    static const uint32_t *d_list[64], *d_index[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return fail_msg("no CUDA device");
    std::lock_guard<std::mutex> lock(mu);
    if (!d_list[dev]) {
        uint32_t *l = nullptr, *ix = nullptr;
        cudaError_t e = cudaMalloc(&l, sizeof l3m_expf_list_host);
        if (e == cudaSuccess) e = cudaMalloc(&ix, sizeof l3m_expf_index_host);
        if (e == cudaSuccess) e = cudaMemcpy(l, l3m_expf_list_host, sizeof l3m_expf_list_host, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ix, l3m_expf_index_host, sizeof l3m_expf_index_host, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail(e, "expf tables");
        d_list[dev] = l;
        d_index[dev] = ix;
    }
    *list = d_list[dev];
    *index = d_index[dev];
    return 0;
}

// Error text for the other entry-point files of this library (not exported).
extern "C" int l3m_error_msg(const char *msg) { return fail_msg(msg); }
extern "C" int l3m_error_cuda(int e, const char *what) { return fail((cudaError_t)e, what); }

extern "C" {

L3M_API const char *l3m_cuda_error(void) { return g_err; }

L3M_API int l3m_gemv_dev(int exact, int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream) {
    if (dtype < 0 || dtype >= L3M_DT_COUNT || ntiles < 0 || k <= 0) return fail_msg("l3m_gemv_dev: bad arguments");
    if (dtype >= DT_Q8 && k % kQB) return fail_msg("l3m_gemv_dev: quantised k must be a multiple of 32");
    if (dtype == DT_BF16 && k % 2) return fail_msg("l3m_gemv_dev: bf16 k must be even");
    if (ntiles == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    if (!exact && dtype <= DT_BF16) {
        gemv_fast_kernel<<<grid_for((ntiles + 15) / 16), kThreads, 0, s>>>(dtype, y, (const uint8_t *)tiles, ntiles, k, vec_arg(x));
    } else {
        const int per_cta = (ntiles + grid_for(ntiles) - 1) / grid_for(ntiles);
        size_t smem = prep_smem(k) + (size_t)kScratchPairs * sizeof(float2) + (size_t)per_cta * kTile * 4;
        if (dtype >= DT_Q8 && (size_t)(k / kQB) * kTile > (size_t)kScratchPairs) return fail_msg("l3m_gemv_dev: k too large");
        cudaError_t e = cudaFuncSetAttribute(gemv_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail(e, "l3m_gemv_dev");
        gemv_exact_kernel<<<grid_for(ntiles), kThreads, smem, s>>>(dtype, y, (const uint8_t *)tiles, ntiles, k, vec_arg(x));
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_gemv_dev");
}

L3M_API int l3m_vec_prepare_dev(int dtype, l3m_vec *out, const float *x, int n, void *scratch, void *stream) {
    if (dtype >= DT_Q8 && n % kQB) return fail_msg("l3m_vec_prepare_dev: n must be a multiple of 32");
    memset(out, 0, sizeof *out);
    out->f32 = x;
    if (dtype == DT_F32) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    int8_t *q = (int8_t *)scratch;
    float *scale = (float *)(q + n);
    int32_t *sum = (int32_t *)(scale + n / kQB);
    int grid = (n + kThreads - 1) / kThreads;
    if (dtype == DT_BF16) {
        prepare_kernel<<<grid, kThreads, 0, s>>>(dtype, x, n, nullptr, nullptr, nullptr, (uint16_t *)scratch);
        out->bf16 = (const uint16_t *)scratch;
    } else {
        prepare_kernel<<<grid, kThreads, 0, s>>>(dtype, x, n, q, scale, sum, nullptr);
        out->q8 = q; out->scale = scale; out->sum = sum;
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_vec_prepare_dev");
}

L3M_API int l3m_block_dots_dev(int dtype, int32_t *dots, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream) {
    if (dtype < DT_Q8 || dtype > DT_MX || k % kQB) return fail_msg("l3m_block_dots_dev: quantised dtypes, k a multiple of 32");
    if (ntiles == 0) return 0;
    block_dots_kernel<<<grid_for(ntiles), 256, 0, (cudaStream_t)stream>>>(dtype, dots, (const uint8_t *)tiles, ntiles, k, vec_arg(x));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_block_dots_dev");
}

L3M_API int l3m_unpack_dev(int dtype, int8_t *q, float *d, const void *tiles, int ntiles, int k, void *stream) {
    if (dtype < DT_Q8 || dtype > DT_MX || k % kQB) return fail_msg("l3m_unpack_dev: quantised dtypes, k a multiple of 32");
    if (ntiles == 0) return 0;
    unpack_kernel<<<grid_for(ntiles), 256, 0, (cudaStream_t)stream>>>(dtype, q, d, (const uint8_t *)tiles, ntiles, k);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_unpack_dev");
}

L3M_API int l3m_attend_dev(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int head_dim, int stride, void *stream) {
    if (head_dim % 8 || head_dim <= 0 || pos < 0 || stride < head_dim) return fail_msg("l3m_attend_dev: bad arguments");
    const uint32_t *list, *index;
    if (l3m_expf_tables(&list, &index)) return -1;
    size_t smem = (size_t)head_dim * 8 + 64 * 4 + (size_t)((pos + 4) & ~3) * 4 + (size_t)head_dim * 4 + 16 +
                  (size_t)kAttnChunk * (head_dim + 8) * 2;
    cudaError_t e = cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(e, "l3m_attend_dev");
    attend_kernel<<<1, kThreads, smem, (cudaStream_t)stream>>>(out, q, k, v, pos, head_dim, stride, list, index);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_attend_dev");
}

}  // extern "C"
