// Device helpers shared by the matvec and decode kernels (sm_100a).
#pragma once
#include <cstdint>
#include "numerics.h"
#include "expf_exact.h"

namespace l3m {

constexpr int kTile = 16;
constexpr int kQB = 32;

// ---- loads
// Weights are read-only for a kernel's lifetime: the non-coherent path, as plain intrinsics so the
// compiler is free to hoist and batch them.
__device__ __forceinline__ uint4 ld_nc_v4(const void *p) { return __ldg((const uint4 *)p); }
__device__ __forceinline__ uint32_t ld_nc_u32(const void *p) { return __ldg((const unsigned int *)p); }
__device__ __forceinline__ uint16_t ld_nc_u16(const void *p) { return __ldg((const unsigned short *)p); }
__device__ __forceinline__ uint8_t ld_nc_u8(const void *p) { return __ldg((const unsigned char *)p); }
// Data other CTAs write during the kernel (KV cache rows): cached in L2 only, never in L1, so a
// line fetched before a neighbouring row was written cannot be served stale.
__device__ __forceinline__ uint4 ld_cg_v4(const void *p) { return __ldcg((const uint4 *)p); }
__device__ __forceinline__ float ld_cg_f32(const float *p) { return __ldcg(p); }
// Streamed read-only data (weights): not allocated in L1, so it does not evict what the kernel reuses.
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void *p) {
    uint2 v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const void *p) {
    uint32_t v;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
// 16-byte asynchronous copy global -> shared through L2 (both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ uint16_t ld_cg_u16(const void *p) { return __ldcg((const unsigned short *)p); }

// ---- integer dot of 4 bytes: unsigned weights times signed activations, plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// ---- exchange slots: one 64-bit word = {float bits (low), epoch (high)}, written and read whole.
// A slot is ready when its epoch equals the expected one; buffers are zeroed before each launch
// and epochs start at 1, so a stale slot never matches. Stores release and polls acquire, so data
// written before a publish (KV cache rows) is visible to every CTA that has seen the slot.
__device__ __forceinline__ uint64_t slot_word(float v, uint32_t epoch) {
    return ((uint64_t)epoch << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void slot_put(uint64_t *s, uint64_t w) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(s), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t slot_get(const uint64_t *s) {
    uint64_t w;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(s) : "memory");
    return w;
}
// System scope: peer GPUs' memory and host-mapped memory.
__device__ __forceinline__ void slot_put_sys(uint64_t *s, uint64_t w) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(s), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t slot_get_sys(const uint64_t *s) {
    uint64_t w;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(s) : "memory");
    return w;
}
__device__ __forceinline__ int ld_relaxed_sys_i32(const int *p) {
    int v;
    asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t slot_epoch(uint64_t w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float slot_value(uint64_t w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- warp reductions (exact: integer sums, max)
__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace l3m
