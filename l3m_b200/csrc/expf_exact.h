// expf that returns, bit for bit, what the host C library's expf returns, written once for both
// the host (the build-time generator) and the device (the decode kernels).
//
// Method: e^x is evaluated in double precision (x = k ln2 + r, |r| <= ln2/2, degree-12 Taylor
// polynomial, scaled by 2^k) and rounded to float. That is correctly rounded except when e^x lies
// within about 2^-47 of a float rounding midpoint. The C library's expf is not always correctly
// rounded; every input where the two differ lies within L3M_EXPF_WINDOW ulp of a midpoint (the
// generator checks this over all 2^32 inputs). So: round the double result, and only when it falls
// inside that window look the input up in the exceptions produced by running the C library (held
// as an open-addressing hash set, so a lookup is usually one memory read); a listed input takes the
// other float neighbour.
//
// Every operation is a single IEEE double operation (multiply, fused multiply-add, rint), so the
// host and the device compute identical values. L3M_EXPF_HD marks functions for both compilers.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define L3M_EXPF_HD __host__ __device__ __forceinline__
#else
#define L3M_EXPF_HD static inline
#include <math.h>
#include <string.h>
#endif

#define L3M_EXPF_WINDOW 0.002   // ulp; the generator asserts every exception lies inside it

L3M_EXPF_HD uint32_t l3m_f2u(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}
L3M_EXPF_HD float l3m_u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f; memcpy(&f, &u, 4); return f;
#endif
}
L3M_EXPF_HD double l3m_u2d(uint64_t u) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)u);
#else
    double d; memcpy(&d, &u, 8); return d;
#endif
}
L3M_EXPF_HD double l3m_fma(double a, double b, double c) {
#ifdef __CUDA_ARCH__
    return __fma_rn(a, b, c);
#else
    return fma(a, b, c);
#endif
}
L3M_EXPF_HD double l3m_mul(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}
L3M_EXPF_HD double l3m_rint(double a) { return rint(a); }

// e^x in double for finite x in [-104, 89].
L3M_EXPF_HD double l3m_exp_double(float xf) {
    double x = (double)xf;
    double k = l3m_rint(l3m_mul(x, 1.4426950408889634));            // 1/ln2
    const double L1 = 0x1.62e42fefa3800p-1, L2 = 0x1.ef35793c7673p-45;   // ln2 = L1 + L2, L1 with trailing zeros
    double r = l3m_fma(-k, L1, x);
    r = l3m_fma(-k, L2, r);
    double p = 1.0 / 479001600.0;                                     // 1/12!
    p = l3m_fma(p, r, 1.0 / 39916800.0);
    p = l3m_fma(p, r, 1.0 / 3628800.0);
    p = l3m_fma(p, r, 1.0 / 362880.0);
    p = l3m_fma(p, r, 1.0 / 40320.0);
    p = l3m_fma(p, r, 1.0 / 5040.0);
    p = l3m_fma(p, r, 1.0 / 720.0);
    p = l3m_fma(p, r, 1.0 / 120.0);
    p = l3m_fma(p, r, 1.0 / 24.0);
    p = l3m_fma(p, r, 1.0 / 6.0);
    p = l3m_fma(p, r, 0.5);
    p = l3m_fma(p, r, 1.0);
    p = l3m_fma(p, r, 1.0);
    int ki = (int)k;                                                  // |k| <= 150: 2^k is a normal double
    return l3m_mul(p, l3m_u2d((uint64_t)(ki + 1023) << 52));
}

// Correctly rounded candidate and whether the exception list must be consulted. *other is the float
// on the far side of the double value (the answer for a listed input).
L3M_EXPF_HD float l3m_expf_candidate(float x, int *check, float *other) {
    *check = 0;
    *other = 0.0f;
    if (x != x) return x + x;                      // NaN
    if (x > 89.0f) return l3m_u2f(0x7F800000u);    // overflow: +inf
    if (x < -104.0f) return 0.0f;                  // underflow: +0
    double y = l3m_exp_double(x);
    float f = (float)y;                            // round to nearest even (subnormals included)
    uint32_t fu = l3m_f2u(f);
    if (fu == 0x7F800000u) return f;
    float lo = f, hi = f;
    if ((double)f > y) lo = fu ? l3m_u2f(fu - 1) : 0.0f; else hi = l3m_u2f(fu + 1);
    if (lo == hi) return f;
    double mid = ((double)lo + (double)hi) * 0.5, ulp = (double)hi - (double)lo;
    double dist = y > mid ? y - mid : mid - y;
    if (dist <= L3M_EXPF_WINDOW * ulp) {
        *check = 1;
        *other = f == hi ? lo : hi;
    }
    return f;
}

// The exception set: 2^L3M_EXPF_HASH_BITS slots of input bit patterns, empty slots L3M_EXPF_EMPTY (a
// NaN pattern, never listed), linear probing from l3m_expf_slot(u); the builder guarantees that every
// probe sequence, for a listed input or not, ends within L3M_EXPF_PROBES slots.
#define L3M_EXPF_HASH_BITS 19
#define L3M_EXPF_SLOTS (1u << L3M_EXPF_HASH_BITS)
#define L3M_EXPF_EMPTY 0xFFFFFFFFu
#define L3M_EXPF_PROBES 64
L3M_EXPF_HD uint32_t l3m_expf_slot(uint32_t u) { return (uint32_t)(u * 0x9E3779B1u) >> (32 - L3M_EXPF_HASH_BITS); }

// One slot. On the device with an L2 evict-last policy (pol): the table is prefetched into L2 with the
// same policy when a decode launch starts, so the rare lookups stay in L2 while the weights stream past.
L3M_EXPF_HD uint32_t l3m_expf_slot_load(const uint32_t *table, uint32_t i, uint64_t pol) {
#ifdef __CUDA_ARCH__
    uint32_t v;
    asm volatile("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(table + i), "l"(pol));
    return v;
#else
    (void)pol;
    return table[i];
#endif
}

L3M_EXPF_HD int l3m_expf_listed(uint32_t u, const uint32_t *table) {
    uint32_t i = l3m_expf_slot(u);
    uint64_t pol = 0;
#ifdef __CUDA_ARCH__
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
#pragma unroll 1
#endif
    for (int p = 0; p < L3M_EXPF_PROBES; p++) {                // kept rolled: the first probe almost always ends it
        const uint32_t v = l3m_expf_slot_load(table, i, pol);
        if (v == u) return 1;
        if (v == L3M_EXPF_EMPTY) return 0;
        i = (i + 1) & (L3M_EXPF_SLOTS - 1);
    }
    return 0;
}

#ifdef __CUDACC__
#define L3M_EXPF_HOST static inline __host__
#else
#define L3M_EXPF_HOST static inline
#endif
// Host: fill table[L3M_EXPF_SLOTS] from the n listed inputs. Returns 0, or -1 when the set does not
// fit (more inputs than half the slots, or a run of occupied slots reaching L3M_EXPF_PROBES).
L3M_EXPF_HOST int l3m_expf_hash_build(const uint32_t *list, size_t n, uint32_t *table) {
    if (n > L3M_EXPF_SLOTS / 2) return -1;
    for (uint32_t i = 0; i < L3M_EXPF_SLOTS; i++) table[i] = L3M_EXPF_EMPTY;
    for (size_t j = 0; j < n; j++) {
        uint32_t i = l3m_expf_slot(list[j]);
        while (table[i] != L3M_EXPF_EMPTY && table[i] != list[j]) i = (i + 1) & (L3M_EXPF_SLOTS - 1);
        table[i] = list[j];
    }
    // Longest run of occupied slots (cyclic): every probe sequence ends at the empty slot after its run.
    uint32_t run = 0, longest = 0, start = 0;
    while (start < L3M_EXPF_SLOTS && table[start] != L3M_EXPF_EMPTY) start++;
    for (uint32_t k = 1; k <= L3M_EXPF_SLOTS; k++) {
        const uint32_t i = (start + k) & (L3M_EXPF_SLOTS - 1);
        run = table[i] == L3M_EXPF_EMPTY ? 0 : run + 1;
        if (run > longest) longest = run;
    }
    return longest + 1 < L3M_EXPF_PROBES ? 0 : -1;
}

L3M_EXPF_HD float l3m_expf_exact(float x, const uint32_t *table) {
    int check; float other;
    float f = l3m_expf_candidate(x, &check, &other);
    if (check && l3m_expf_listed(l3m_f2u(x), table)) return other;
    return f;
}
