// The host-pointer kernel tables and their selection (replaces reference src/dispatch.c:1-36 and the
// per-ISA tables of src/kernels_*.c). A table entry copies its inputs to the current device, runs
// the device kernel and copies y back: the reference's l3m_gemv_fn contract, served by the GPU.
// That contract has no error return: when a copy or launch fails, the entry prints the reason on
// stderr and fills its output with NaN, so a failed call cannot pass for a result.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include "../../include/l3m_kernels.h"

extern "C" int l3m_expf_table(const uint32_t **table);

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_buf[kMaxDevices];
size_t g_cap[kMaxDevices];

// The current device's staging buffer, grown on demand (one per device: a kernel reads only its own
// device's memory). Called with g_mu held.
void *scratch(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    if (bytes <= g_cap[dev]) return g_buf[dev];
    if (g_buf[dev]) cudaFree(g_buf[dev]);
    g_buf[dev] = nullptr;
    g_cap[dev] = 0;
    if (cudaMalloc(&g_buf[dev], bytes) != cudaSuccess) return nullptr;
    g_cap[dev] = bytes;
    return g_buf[dev];
}

size_t up(size_t n) { return (n + 255) & ~(size_t)255; }

bool put(void *dst, const void *src, size_t n) { return cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice) == cudaSuccess; }

void fail_nan(const char *what, const char *why, float *out, size_t n) {
    fprintf(stderr, "l3m: %s: %s\n", what, why);
    for (size_t i = 0; i < n; i++) out[i] = __builtin_nanf("");
}

void shim(int exact, int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x) {
    std::lock_guard<std::mutex> lock(g_mu);
    const size_t tb = (size_t)ntiles * l3m_tile_bytes(dtype, k), yb = (size_t)ntiles * L3M_TILE * 4;
    const size_t xb = (size_t)k * 4 + (size_t)k * 2 + (size_t)k + (size_t)(k / 32 + 1) * 8;
    char *d = (char *)scratch(up(tb) + up(yb) + up(xb) + 1024);
    if (!d) return fail_nan("gemv", "device allocation failed", y, yb / 4);
    char *dt = d, *dy = d + up(tb), *dx = dy + up(yb);
    l3m_vec v = {};
    bool ok = put(dt, tiles, tb);
    if (dtype == L3M_DT_F32) {
        ok = ok && put(dx, x->f32, (size_t)k * 4);
        v.f32 = (const float *)dx;
    } else if (dtype == L3M_DT_BF16) {
        ok = ok && put(dx, x->bf16, (size_t)k * 2);
        v.bf16 = (const uint16_t *)dx;
    } else {
        int8_t *q = (int8_t *)dx;
        float *sc = (float *)(dx + up(k));
        int32_t *su = (int32_t *)(dx + up(k) + up((size_t)(k / 32) * 4));
        ok = ok && put(q, x->q8, (size_t)k) && put(sc, x->scale, (size_t)(k / 32) * 4) && put(su, x->sum, (size_t)(k / 32) * 4);
        v.q8 = q; v.scale = sc; v.sum = su;
    }
    if (!ok) return fail_nan("gemv", "copy to the device failed", y, yb / 4);
    if (l3m_gemv_dev(exact, dtype, (float *)dy, dt, ntiles, k, &v, nullptr)) return fail_nan("gemv", l3m_cuda_error(), y, yb / 4);
    cudaError_t e = cudaMemcpy(y, dy, yb, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) fail_nan("gemv", cudaGetErrorString(e), y, yb / 4);
}

template <int DT> void gemv_exact(float *y, const void *t, int n, int k, const l3m_vec *x) { shim(1, DT, y, t, n, k, x); }
template <int DT> void gemv_fast(float *y, const void *t, int n, int k, const l3m_vec *x) { shim(0, DT, y, t, n, k, x); }

void attend_shim(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int hd, int stride) {
    std::lock_guard<std::mutex> lock(g_mu);
    const size_t kvb = ((size_t)pos * stride + hd) * 2;
    char *d = (char *)scratch(up(kvb) * 2 + up((size_t)hd * 4) * 2 + 1024);
    if (!d) return fail_nan("attend", "device allocation failed", out, (size_t)hd);
    char *dk = d, *dv = d + up(kvb), *dq = dv + up(kvb), *dout = dq + up((size_t)hd * 4);
    if (!put(dk, k, kvb) || !put(dv, v, kvb) || !put(dq, q, (size_t)hd * 4)) return fail_nan("attend", "copy to the device failed", out, (size_t)hd);
    if (l3m_attend_dev((float *)dout, (const float *)dq, (const uint16_t *)dk, (const uint16_t *)dv, pos, hd, stride, nullptr))
        return fail_nan("attend", l3m_cuda_error(), out, (size_t)hd);
    cudaError_t e = cudaMemcpy(out, dout, (size_t)hd * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) fail_nan("attend", cudaGetErrorString(e), out, (size_t)hd);
}

}  // namespace

extern "C" {

L3M_API const l3m_kernels l3m_kernels_sm100a = {
    "sm100a",
    {gemv_exact<L3M_DT_F32>, gemv_exact<L3M_DT_BF16>, gemv_exact<L3M_DT_Q8_0>, gemv_exact<L3M_DT_Q4_0>, gemv_exact<L3M_DT_MXFP4>},
    attend_shim,
};

L3M_API const l3m_kernels l3m_kernels_sm100a_fast = {
    "sm100a-fast",
    {gemv_fast<L3M_DT_F32>, gemv_fast<L3M_DT_BF16>, gemv_exact<L3M_DT_Q8_0>, gemv_exact<L3M_DT_Q4_0>, gemv_exact<L3M_DT_MXFP4>},
    attend_shim,
};

L3M_API int l3m_kernels_usable(const l3m_kernels *k) {
    if (k != &l3m_kernels_sm100a && k != &l3m_kernels_sm100a_fast) return 0;
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
    return major == 10;
}

L3M_API const l3m_kernels *l3m_kernels_pick(void) {
    const char *want = getenv("L3M_ISA");
    if (!want || !strcmp(want, "sm100a")) return &l3m_kernels_sm100a;
    if (!strcmp(want, "sm100a-fast")) return &l3m_kernels_sm100a_fast;
    fprintf(stderr, "l3m: L3M_ISA=%s not available here, using sm100a\n", want);
    return &l3m_kernels_sm100a;
}

}  // extern "C"
