// l3m_gemv_splitk_dev: the exact quantised matvec with its K dimension split across the whole GPU,
// for callers that cannot allocate device memory. The per-(output, 32-input block) results live in
// one fixed static device buffer of this file instead of memory the call would allocate.
//
// Pass 1 (splitk_dots): one thread per (output, block) item over every SM computes the exact
// integer block dot and stores {RN(sx[b] * d), (float)dot} at scratch[b * n_out + o].
// Pass 2 (splitk_chain): one thread per output runs the fp32 chain acc = fma(s, dot, acc) over the
// blocks in order — the order of the reference's scalar kernels (src/kernels_scalar.c:30-75) — so
// y equals l3m_gemv_dev's exact table bit for bit. Both passes run on the caller's stream, in order.
//
// Limits and rules:
//  - quantised dtypes only (q8_0, q4_0, mxfp4): the f32/bf16 chains run over single inputs and do
//    not split;
//  - at most kSplitKMaxPairs = 524,288 block results per call (ntiles * 16 * k/32; 4 MiB): larger
//    calls are rejected before anything is launched;
//  - nothing in the scratch needs to start at zero: pass 2 reads only what pass 1 of the same
//    call wrote;
//  - the scratch is one buffer per device and per process: calls that overlap on one device (two
//    streams, two host threads) race on it and must be serialised by the caller;
//  - the first call on each device looks up the buffer's address (cudaGetSymbolAddress, which may
//    load this library's device code); that address is kept for the life of the process: it belongs to the device's context of the
//    first call, so a device reset (cudaDeviceReset, or a reset of the primary context) while this
//    library is loaded leaves it stale; do not reset a device that this entry point has used;
//  - misaligned pointers (tiles, y, and x's q8, scale and sum must be 4-byte aligned) are refused
//    before anything launches, like every other bad argument.
#include <cuda_runtime.h>
#include <cstdio>
#include <mutex>
#include "ops.cuh"
#include "../../include/l3m_kernels.h"

using namespace l3m;

extern "C" int l3m_error_msg(const char *msg);
extern "C" int l3m_error_cuda(int e, const char *what);

namespace {

constexpr long long kSplitKMaxPairs = 1 << 19;
constexpr int kMaxDevices = 64;
constexpr int kThreads = 256;

static __device__ __align__(256) float2 g_splitk_scratch[kSplitKMaxPairs];

struct DeviceSlot { float2 *scratch; int sms; };
std::mutex g_mu;
DeviceSlot g_slots[kMaxDevices];

// Once per device, with that device current: the scratch buffer's address and the SM count.
int setup(DeviceSlot *out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return l3m_error_cuda(e, "l3m_gemv_splitk_dev: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return l3m_error_msg("l3m_gemv_splitk_dev: device ordinal beyond 63");
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceSlot &s = g_slots[dev];
    if (!s.scratch) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_splitk_scratch);
        if (e != cudaSuccess) return l3m_error_cuda(e, "l3m_gemv_splitk_dev: cudaGetSymbolAddress(scratch)");
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return l3m_error_cuda(e, "l3m_gemv_splitk_dev: SM count");
        s.sms = sms > 0 ? sms : 148;
        s.scratch = (float2 *)p;
    }
    *out = s;
    return 0;
}

template <int DT>
__global__ void __launch_bounds__(kThreads) splitk_dots(float2 *__restrict__ scratch, const uint8_t *__restrict__ tiles, int n_out, int nb,
                                                         const int8_t *__restrict__ xq, const float *__restrict__ xscale,
                                                         const int32_t *__restrict__ xsum) {
    const int bb = block_bytes(DT);
    const size_t tb = (size_t)nb * bb;
    const long long items = (long long)n_out * nb;
    const uint32_t *xw = (const uint32_t *)xq;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / n_out), o = (int)(i - (long long)b * n_out);
        QLoad q;
        qload<DT>(q, tiles + (size_t)(o >> 4) * tb + (size_t)b * bb, o & 15);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = __ldg(xw + 8 * b + j);
        const int dot = qdot<DT>(q, w, __ldg(xsum + b));
        scratch[i] = make_float2(__fmul_rn(__ldg(xscale + b), qscale<DT>(q.d)), __int2float_rn(dot));
    }
}

__global__ void __launch_bounds__(kThreads) splitk_chain(float *__restrict__ y, const float2 *__restrict__ scratch, int n_out, int nb) {
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= n_out) return;
    float acc = 0.0f;
#pragma unroll 4
    for (int b = 0; b < nb; b++) {
        const float2 v = scratch[(size_t)b * n_out + o];
        acc = __fmaf_rn(v.x, v.y, acc);
    }
    y[o] = acc;
}

}  // namespace

extern "C" L3M_API int l3m_gemv_splitk_dev(int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream) {
    if (dtype < L3M_DT_Q8_0 || dtype > L3M_DT_MXFP4)
        return l3m_error_msg("l3m_gemv_splitk_dev: quantised dtypes only (q8_0, q4_0, mxfp4); use l3m_gemv_dev for f32/bf16");
    if (ntiles < 0 || k <= 0 || k % kQB) return l3m_error_msg("l3m_gemv_splitk_dev: bad arguments (k a positive multiple of 32, ntiles >= 0)");
    const long long n_out = (long long)ntiles * kTile, nb = k / kQB, pairs = n_out * nb;
    if (pairs > kSplitKMaxPairs) {
        char msg[200];
        snprintf(msg, sizeof msg, "l3m_gemv_splitk_dev: ntiles*16*(k/32) = %lld block results exceed the static scratch of %lld; use l3m_gemv_dev",
                 pairs, kSplitKMaxPairs);
        return l3m_error_msg(msg);
    }
    if (ntiles == 0) return 0;
    if (!y || !tiles || !x || !x->q8 || !x->scale || !x->sum)
        return l3m_error_msg("l3m_gemv_splitk_dev: y, tiles and a prepared x (q8, scale, sum) are required");
    if (((uintptr_t)tiles | (uintptr_t)y | (uintptr_t)x->q8 | (uintptr_t)x->scale | (uintptr_t)x->sum) & 3)
        return l3m_error_msg("l3m_gemv_splitk_dev: tiles, y, q8, scale and sum must be 4-byte aligned");
    DeviceSlot slot;
    if (setup(&slot)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    long long blocks = (pairs + kThreads - 1) / kThreads, cap = 8LL * slot.sms;
    const int g1 = (int)(blocks < cap ? blocks : cap), g2 = (int)((n_out + kThreads - 1) / kThreads);
    const uint8_t *t = (const uint8_t *)tiles;
    if (dtype == L3M_DT_Q8_0) splitk_dots<DT_Q8><<<g1, kThreads, 0, s>>>(slot.scratch, t, (int)n_out, (int)nb, x->q8, x->scale, x->sum);
    else if (dtype == L3M_DT_Q4_0) splitk_dots<DT_Q4><<<g1, kThreads, 0, s>>>(slot.scratch, t, (int)n_out, (int)nb, x->q8, x->scale, x->sum);
    else splitk_dots<DT_MX><<<g1, kThreads, 0, s>>>(slot.scratch, t, (int)n_out, (int)nb, x->q8, x->scale, x->sum);
    splitk_chain<<<g2, kThreads, 0, s>>>(y, slot.scratch, (int)n_out, (int)nb);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : l3m_error_cuda(e, "l3m_gemv_splitk_dev");
}
