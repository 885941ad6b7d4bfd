// ORACLE — test infrastructure only (see oracle.h).
#include <math.h>
#include "oracle.h"

// The reference calls the C library's expf (reference src/ops.c:45, 50); so does the oracle.
float o_expf(float x) { return expf(x); }

// The C library's expf over n values (a device expf is checked against this, bit for bit).
void o_expf_n(const float *x, float *y, int n) {
    for (int i = 0; i < n; i++) y[i] = expf(x[i]);
}
