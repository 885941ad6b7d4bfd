// The host-pointer kernel tables and their selection (replaces reference src/dispatch.c:1-36 and the
// per-ISA tables of src/kernels_*.c). A table entry copies its inputs to the current device, runs
// the device kernel and copies y back: the reference's l3m_gemv_fn contract, served by the GPU.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include "../../include/l3m_kernels.h"

extern "C" int l3m_expf_tables(const uint32_t **list, const uint32_t **index);

namespace {

std::mutex g_mu;
void *g_buf = nullptr;
size_t g_cap = 0;

void *scratch(size_t bytes) {                         // one device staging buffer, grown on demand
    if (bytes <= g_cap) return g_buf;
    if (g_buf) cudaFree(g_buf);
    g_buf = nullptr;
    g_cap = 0;
    if (cudaMalloc(&g_buf, bytes) != cudaSuccess) return nullptr;
    g_cap = bytes;
    return g_buf;
}

size_t up(size_t n) { return (n + 255) & ~(size_t)255; }

void shim(int exact, int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x) {
    std::lock_guard<std::mutex> lock(g_mu);
    const size_t tb = (size_t)ntiles * l3m_tile_bytes(dtype, k), yb = (size_t)ntiles * L3M_TILE * 4;
    const size_t xb = (size_t)k * 4 + (size_t)k * 2 + (size_t)k + (size_t)(k / 32 + 1) * 8;
    char *d = (char *)scratch(up(tb) + up(yb) + up(xb) + 1024);
    if (!d) { fprintf(stderr, "l3m: gemv: device allocation failed\n"); return; }
    char *dt = d, *dy = d + up(tb), *dx = dy + up(yb);
    l3m_vec v = {};
    cudaMemcpy(dt, tiles, tb, cudaMemcpyHostToDevice);
    if (dtype == L3M_DT_F32) {
        cudaMemcpy(dx, x->f32, (size_t)k * 4, cudaMemcpyHostToDevice);
        v.f32 = (const float *)dx;
    } else if (dtype == L3M_DT_BF16) {
        cudaMemcpy(dx, x->bf16, (size_t)k * 2, cudaMemcpyHostToDevice);
        v.bf16 = (const uint16_t *)dx;
    } else {
        int8_t *q = (int8_t *)dx;
        float *sc = (float *)(dx + up(k));
        int32_t *su = (int32_t *)(dx + up(k) + up((size_t)(k / 32) * 4));
        cudaMemcpy(q, x->q8, (size_t)k, cudaMemcpyHostToDevice);
        cudaMemcpy(sc, x->scale, (size_t)(k / 32) * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(su, x->sum, (size_t)(k / 32) * 4, cudaMemcpyHostToDevice);
        v.q8 = q; v.scale = sc; v.sum = su;
    }
    if (l3m_gemv_dev(exact, dtype, (float *)dy, dt, ntiles, k, &v, nullptr)) {
        fprintf(stderr, "l3m: gemv: %s\n", l3m_cuda_error());
        return;
    }
    cudaError_t e = cudaMemcpy(y, dy, yb, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) fprintf(stderr, "l3m: gemv: %s\n", cudaGetErrorString(e));
}

template <int DT> void gemv_exact(float *y, const void *t, int n, int k, const l3m_vec *x) { shim(1, DT, y, t, n, k, x); }
template <int DT> void gemv_fast(float *y, const void *t, int n, int k, const l3m_vec *x) { shim(0, DT, y, t, n, k, x); }

void attend_shim(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int hd, int stride) {
    std::lock_guard<std::mutex> lock(g_mu);
    const size_t kvb = ((size_t)pos * stride + hd) * 2;
    char *d = (char *)scratch(up(kvb) * 2 + up((size_t)hd * 4) * 2 + 1024);
    if (!d) { fprintf(stderr, "l3m: attend: device allocation failed\n"); return; }
    char *dk = d, *dv = d + up(kvb), *dq = dv + up(kvb), *dout = dq + up((size_t)hd * 4);
    cudaMemcpy(dk, k, kvb, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, v, kvb, cudaMemcpyHostToDevice);
    cudaMemcpy(dq, q, (size_t)hd * 4, cudaMemcpyHostToDevice);
    if (l3m_attend_dev((float *)dout, (const float *)dq, (const uint16_t *)dk, (const uint16_t *)dv, pos, hd, stride, nullptr)) {
        fprintf(stderr, "l3m: attend: %s\n", l3m_cuda_error());
        return;
    }
    cudaMemcpy(out, dout, (size_t)hd * 4, cudaMemcpyDeviceToHost);
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
