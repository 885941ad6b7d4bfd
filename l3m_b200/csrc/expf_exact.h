// expf that returns, bit for bit, what the host C library's expf returns, written once for both
// the host (the build-time generator) and the device (the decode kernels).
//
// Method: the table-driven evaluation that glibc's expf publishes (since glibc 2.28; ARM's optimized
// routines), restated in double precision: z = x N/ln2 (N = 32) split as k + r with the shift trick,
// |r| <= 1/2; e^x = 2^(k/N) 2^(r/N) with 2^((k mod N)/N) from a 32-entry table of correctly rounded
// doubles scaled by 2^floor(k/N), and 2^(r/N) - 1 by a cubic; the double result rounded to float. The
// first step is one fused multiply-add (as x86-64 builds of the C library with FMA evaluate it). On
// this method the C library and this code agree on every input (the generator checks all 2^32 at build
// time). For a C library that differs, the same check collects the inputs where it does: each must lie
// within L3M_EXPF_WINDOW ulp of a float rounding midpoint of the double result, and those inputs, held
// as an open-addressing hash set, take the other float neighbour. With an empty set (this method's own
// library) the kernels get no table and never look anything up.
//
// Every operation is a single IEEE double operation (multiply, add, fused multiply-add, conversion), so
// the host and the device compute identical values. L3M_EXPF_HD marks functions for both compilers.
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
L3M_EXPF_HD double l3m_sub(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dsub_rn(a, b);
#else
    return a - b;
#endif
}
L3M_EXPF_HD uint64_t l3m_d2u(double d) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u; memcpy(&u, &d, 8); return u;
#endif
}

// 2^(i/32), i = 0..31, each the double nearest to it.
#define L3M_EXP2_TAB {                                                                                    \
    0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,                \
    0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,                \
    0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,                \
    0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,                \
    0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,                \
    0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,                \
    0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,                \
    0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0}
static const double l3m_exp2_tab_host[32] = L3M_EXP2_TAB;
#ifdef __CUDACC__
static __device__ const double l3m_exp2_tab_dev[32] = L3M_EXP2_TAB;
#endif
L3M_EXPF_HD double l3m_exp2_tab(int i) {
#ifdef __CUDA_ARCH__
    return __ldg(&l3m_exp2_tab_dev[i]);
#else
    return l3m_exp2_tab_host[i];
#endif
}

// e^x in double for finite x in [-0x1.9fe368p6, 0x1.62e42ep6] (the float results from 0 to the
// largest float): the method above.
L3M_EXPF_HD double l3m_exp_double(float xf) {
    const double InvLn2N = 0x1.71547652b82fep+0 * 32, Shift = 0x1.8p+52;   // 32/ln2; 1.5 * 2^52
    const double C0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, C1 = 0x1.ebfce50fac4f3p-3 / 32 / 32, C2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double x = (double)xf;
    double kd = l3m_fma(InvLn2N, x, Shift);                          // k in kd's low mantissa bits, rounded to nearest even
    const uint64_t ki = l3m_d2u(kd);
    kd = l3m_sub(kd, Shift);
    const double r = l3m_fma(InvLn2N, x, -kd);                       // |r| <= 1/2
    const int64_t k = (int64_t)(ki << 12) >> 12;                     // the 52-bit field, sign-extended
    const double s = l3m_u2d(l3m_d2u(l3m_exp2_tab((int)(k & 31))) + ((uint64_t)(k >> 5) << 52));   // 2^(k/32), a normal double
    const double z = l3m_fma(C0, r, C1), r2 = l3m_mul(r, r);
    double y = l3m_fma(C2, r, 1.0);
    y = l3m_fma(z, r2, y);
    return l3m_mul(y, s);
}

// Correctly rounded candidate and whether the exception list must be consulted. *other is the float
// on the far side of the double value (the answer for a listed input).
L3M_EXPF_HD float l3m_expf_candidate(float x, int *check, float *other) {
    *check = 0;
    *other = 0.0f;
    if (x != x) return x + x;                      // NaN
    if (x > 0x1.62e42ep6f) return l3m_u2f(0x7F800000u);    // overflow: +inf
    if (x < -0x1.9fe368p6f) return 0.0f;           // underflow: +0
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

// table: the exception set, or null when it is empty (nothing to look up).
L3M_EXPF_HD float l3m_expf_exact(float x, const uint32_t *table) {
    int check; float other;
    float f = l3m_expf_candidate(x, &check, &other);
    if (check && table && l3m_expf_listed(l3m_f2u(x), table)) return other;
    return f;
}
