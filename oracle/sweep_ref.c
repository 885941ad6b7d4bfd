// Test and benchmark infrastructure only: the CPU baseline of the matvec sweep. It times the
// reference's own kernels (l3m_kernels_pick()->gemv[dtype], reference src/kernels.h:33-45) on packed
// sweep tiles, with the tiles split contiguously over an l3m_pool of n cores (reference
// src/pool.h:8-12) and one l3m_sync after every matvec, the way the reference engine runs a sharded
// matvec (src/engine.c:219-223). Built by oracle/Makefile into _ref/libsweep_ref.so, linked against
// the reference objects; only bench.py's CPU-baseline leg and tests/ load it.
#include <stdint.h>
#include <stdlib.h>
#include "kernels.h"
#include "perf.h"
#include "pool.h"

typedef struct {
    l3m_gemv_fn f;
    const uint8_t *tiles;
    size_t tile_bytes;
    int ntiles, k, n, reps;
    const l3m_vec *x;
    float *y;
    double ns;
} sweep_job;

static void sweep_run(l3m_pool *p, int rank, void *arg) {
    sweep_job *j = arg;
    const int t0 = (int)((long)j->ntiles * rank / j->n), t1 = (int)((long)j->ntiles * (rank + 1) / j->n);
    if (t1 > t0) j->f(j->y + (size_t)t0 * 16, j->tiles + (size_t)t0 * j->tile_bytes, t1 - t0, j->k, j->x);   // warm
    l3m_sync(p, rank);
    const double start = l3m_now_ns();
    for (int r = 0; r < j->reps; r++) {
        if (t1 > t0) j->f(j->y + (size_t)t0 * 16, j->tiles + (size_t)t0 * j->tile_bytes, t1 - t0, j->k, j->x);
        l3m_sync(p, rank);
    }
    if (rank == 0) j->ns = (l3m_now_ns() - start) / j->reps;
}

// ns per matvec y[ntiles * 16] = tiles (dtype, k) . x over cores cpus[0..n), averaged over reps;
// the activation is prepared once (l3m_vec_prepare), outside the timing. *table: the kernel table's
// name. Returns -1 if the pool cannot start or the dtype is not in the table.
double sweep_ref_gemv(int dtype, const void *tiles, int ntiles, int k, const float *x, float *y, const int *cpus, int n, int reps,
                      const char **table) {
    const l3m_kernels *kk = l3m_kernels_pick();
    if (table) *table = kk->name;
    if (dtype < 0 || dtype >= L3M_NDTYPES || !kk->gemv[dtype] || n < 1 || reps < 1) return -1;
    void *scratch = malloc((size_t)k * 4 + 64);
    l3m_pool *p = scratch ? l3m_pool_start(cpus, n) : NULL;
    if (!p) { free(scratch); return -1; }
    l3m_vec v;
    l3m_vec_prepare(&v, dtype, x, k, scratch);
    sweep_job j = {kk->gemv[dtype], tiles, l3m_tile_bytes(dtype, k), ntiles, k, n, reps, &v, y, 0.0};
    l3m_pool_run(p, sweep_run, &j);
    l3m_pool_stop(p);
    free(scratch);
    return j.ns;
}
