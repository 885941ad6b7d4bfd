// Scalar conversions shared by the host code and the device kernels, each exact and identical to
// the reference's (src/ops.h:5-6, src/ops.c:5-11, src/pack.c:35-42, src/kernels.h:19-21).
#pragma once
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define L3M_HD __host__ __device__ __forceinline__
#else
#define L3M_HD static inline
#endif

L3M_HD float l3m_bits_f32(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f; memcpy(&f, &u, 4); return f;
#endif
}
L3M_HD uint32_t l3m_f32_bits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}

// bf16 is the top half of an fp32; rounding is to nearest even on the dropped half, with no NaN
// special case (a NaN may round to another NaN or to inf, as in the reference).
L3M_HD float l3m_bf16_to_f32(uint16_t h) { return l3m_bits_f32((uint32_t)h << 16); }
L3M_HD uint16_t l3m_f32_to_bf16(float f) {
    uint32_t u = l3m_f32_bits(f);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// binary16 -> binary32, exact (subnormals scaled by 2^-24, inf and NaN payloads kept). On the
// device the hardware widening (exact for every non-NaN input) with the NaN bits selected, no branch.
L3M_HD float l3m_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
#ifdef __CUDA_ARCH__
    float f;
    asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
    return e == 31 && m ? l3m_bits_f32(sign | 0x7F800000u | m << 13) : f;
#else
    if (e == 0) {
        float mag = (float)m * l3m_bits_f32(0x33800000u);     // m * 2^-24, exact
        return sign ? -mag : mag;
    }
    return l3m_bits_f32(e == 31 ? (sign | 0x7F800000u | m << 13) : (sign | (e + 112u) << 23 | m << 13));
#endif
}

// The mxfp4 block scale of the reference's kernels: 2^(e-127) / 2 = 2^(e-128), subnormal for e < 2.
L3M_HD float l3m_e8m0_half(uint8_t e) {
    return e >= 2 ? l3m_bits_f32((uint32_t)(e - 1) << 23) : l3m_bits_f32(0x00200000u << e);
}

// Doubled e2m1 values by nibble (sign in bit 3), and the same + 16 (all positive).
L3M_HD int l3m_mxfp4_value(int nib) {
    const int mag = (0xC8643210u >> (4 * (nib & 7))) & 15;          // 0 1 2 3 4 6 8 12
    return nib & 8 ? -mag : mag;
}
