// ORACLE — test infrastructure only (see oracle.h).
#include <math.h>
#include "oracle.h"

// The reference calls the C library's expf (reference src/ops.c:45, 50); so does the oracle.
float o_expf(float x) { return expf(x); }

// e^x in double for a float x: x = k*ln2 + r with |r| <= ln2/2 (ln2 split in two so k*L1 is exact),
// a degree-12 Taylor polynomial in Horner form with explicit fma, then 2^k. Relative error below
// 2^-47 over the float range, so rounding the result to float is correctly rounded except within a
// tiny window around float midpoints. The GPU evaluates exactly this sequence of IEEE double
// operations, so both sides agree bit-for-bit; the build step lists the inputs where the host libm's
// expf differs from this correctly rounded value (l3m_b200/csrc/gen_expf_exceptions.c).
double o_exp_double(float xf) {
    double x = xf;
    double k = rint(x * 1.4426950408889634);
    const double L1 = 0x1.62e42fefa3800p-1, L2 = 0x1.ef35793c7673p-45;
    double r = fma(-k, L1, x);
    r = fma(-k, L2, r);
    static const double c[13] = {1.0 / 479001600.0, 1.0 / 39916800.0, 1.0 / 3628800.0, 1.0 / 362880.0, 1.0 / 40320.0,
                                 1.0 / 5040.0, 1.0 / 720.0, 1.0 / 120.0, 1.0 / 24.0, 1.0 / 6.0, 0.5, 1.0, 1.0};
    double p = c[0];
    for (int i = 1; i < 13; i++) p = fma(p, r, c[i]);
    return ldexp(p, (int)k);
}
