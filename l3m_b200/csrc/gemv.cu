// Standalone matvec kernels behind include/l3m_kernels.h: y = tiles . x on the device, with the
// reference's tile layout (src/kernels.h:1-10) and its scalar table's results (src/kernels_scalar.c).
//
// Exact table, quantised dtypes: every CTA takes a contiguous run of tiles; each thread computes the
// exact integer dots of 4 outputs x one 32-input block with dp4a from 16-byte loads (two such items
// in flight), then one thread per output runs the fp32 epilogue over the blocks in order.
// Exact table, f32/bf16: one thread per output runs the sequential chain over K (the order the
// reference rounds in). Fast table, f32/bf16: the chain is split over K across a warp and reduced
// with shuffles (reassociated, like the reference's AVX tables; tolerance-checked).
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>
#include "ops.cuh"
#include "../../include/l3m_kernels.h"

using namespace l3m;

namespace {

thread_local char g_err[256];

int fail(cudaError_t e, const char *what) {
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return -1;
}
int fail_msg(const char *msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return -1;
}

constexpr int kThreads = 512;
constexpr int kScratchPairs = 4096;                 // 32 KB of block results per chunk
constexpr int kAttnChunk = 128;                     // KV rows staged in shared memory at a time

struct VecArg { const float *f32; const uint16_t *bf16; const int8_t *q8; const float *scale; const int32_t *sum; };

__host__ __device__ size_t prep_smem(int k) {                            // q8[k], scale[k/32], sum[k/32], xf[k], 16-byte aligned parts
    size_t a = ((size_t)k + 15) & ~(size_t)15, s = (((size_t)(k / 32 + 1)) * 4 + 15) & ~(size_t)15;
    return a + 2 * s + (size_t)k * 4;
}

__device__ Prep carve_prep(unsigned char *base, int k) {
    Prep p;
    size_t a = ((size_t)k + 15) & ~(size_t)15, s = (((size_t)(k / 32 + 1)) * 4 + 15) & ~(size_t)15;
    p.q8 = (int8_t *)base;
    p.scale = (float *)(base + a);
    p.sum = (int32_t *)(base + a + s);
    p.xf = (float *)(base + a + 2 * s);
    return p;
}

// Copy a prepared vector from global memory into the CTA's shared memory.
__device__ void load_prep(int dtype, const VecArg &x, int k, const Prep &p) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (dtype == DT_F32) for (int i = tid; i < k; i += nth) p.xf[i] = x.f32[i];
    else if (dtype == DT_BF16) for (int i = tid; i < k; i += nth) p.xf[i] = l3m_bf16_to_f32(x.bf16[i]);
    else {
        for (int i = tid; i < k; i += nth) p.q8[i] = x.q8[i];
        for (int i = tid; i < k / 32; i += nth) { p.scale[i] = x.scale[i]; p.sum[i] = x.sum[i]; }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads) gemv_exact_kernel(int dtype, float *y, const uint8_t *tiles, int ntiles, int k, VecArg x) {
    extern __shared__ __align__(16) unsigned char smem[];
    Prep p = carve_prep(smem, k);
    float2 *scratch = (float2 *)(smem + prep_smem(k));
    load_prep(dtype, x, k, p);
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x), t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    float *ys = (float *)(scratch + kScratchPairs);                    // this CTA's outputs, then to global
    matvec_exact(dtype, tiles, k, t0, t1, p, scratch, kScratchPairs, ys);
    for (int o = threadIdx.x; o < (t1 - t0) * kTile; o += blockDim.x) y[(size_t)t0 * kTile + o] = ys[o];
}

// ---- Streamed exact matvec (q8_0, q4_0, mxfp4, bf16 with k a multiple of 32).
// One CTA per SM takes a contiguous run of tiles [t0, t1) and handles it in waves of G tiles; a wave
// reads its tiles' 32-input blocks in order, U blocks per chunk, through a ring of kStreamStages
// shared-memory buffers. A producer warp starts each chunk with one cp.async.bulk per tile (global ->
// this CTA's shared memory, no multicast; bytes complete on the buffer's "full" mbarrier) once the 8
// compute warps have each arrived on the buffer's "empty" mbarrier for its previous chunk, so the
// compute warps never wait for one another inside a wave. Quantised dtypes: each (4 outputs x 1
// block) item leaves {RN(sx*d), (float)dot} in the wave's scratch; at the end of the wave one thread
// per output runs acc = fma(RN(sx*d), dot, acc) over all blocks in order. bf16: each output's thread
// runs the input-order chain straight from the staged words, its accumulator kept across chunks. So
// the rounding sequence is the scalar kernel's (src/kernels_scalar.c:19-75), as in gemv_exact_kernel.
constexpr int kStreamWarps = 8;                     // compute warps; warp 8 produces
constexpr int kStreamThreads = 32 * (kStreamWarps + 1);
constexpr int kStreamStages = 4;
constexpr int kStreamChunk = 32768;                 // target weight bytes per chunk
constexpr int kStreamScratch = 48 * 1024;           // bytes of per-wave (scale product, dot) pairs
constexpr int kConstTiles = 2;                      // l3m_gemv_dev flag: no earlier work on the stream writes the tiles

struct StreamPlan { int G, U, piece, stage_bytes, scratch_pairs, early; };   // early: start the weight copies before the grid dependency

__host__ __device__ inline int stream_unit_bytes(int dtype) { return dtype == DT_BF16 ? 1024 : block_bytes(dtype); }

// tiles_per_cta: the largest run a CTA gets. G: a power of two <= 16 that fits the run (and, for the
// quantised dtypes, whose pairs fit the scratch); U: blocks per chunk so that a chunk is about
// kStreamChunk bytes; piece: a tile's share of a stage buffer, padded by 64 bytes so that
// consecutive tiles start in different bank halves. G = 0: the shape does not fit this kernel.
StreamPlan stream_plan(int dtype, int k, int tiles_per_cta) {
    StreamPlan pl;
    const int bb = stream_unit_bytes(dtype), nb = k / kQB;
    const long long pair_bytes_per_tile = (long long)nb * kTile * sizeof(float2);
    pl.G = 1;
    while (pl.G < 16 && 2 * pl.G <= tiles_per_cta && (dtype == DT_BF16 || 2 * pl.G * pair_bytes_per_tile <= kStreamScratch)) pl.G *= 2;
    if (dtype != DT_BF16 && pair_bytes_per_tile > kStreamScratch) pl.G = 0;
    const int g = pl.G ? pl.G : 1;
    pl.U = std::max(1, std::min(nb, kStreamChunk / (g * bb)));
    pl.piece = pl.U * bb + 64;
    pl.stage_bytes = g * pl.piece;
    pl.scratch_pairs = dtype == DT_BF16 ? 0 : g * nb * kTile;
    pl.early = 0;
    return pl;
}

size_t stream_smem(int k, const StreamPlan &pl) {
    return ((prep_smem(k) + 127) & ~(size_t)127) + (size_t)kStreamStages * pl.stage_bytes + (size_t)pl.scratch_pairs * sizeof(float2);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Wait for phase parity `par` of the mbarrier at shared address bar (time-limited: 2 s). A wait that
// gives up (never expected) marks the CTA failed (*fail: its outputs are written as NaN) and counts
// itself in *timeouts, host-mapped memory that the next l3m_gemv_dev call reports as an error.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t par, int *fail, int *timeouts) {
    uint64_t start = 0;
    for (int spin = 0;; spin++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\tselp.u32 %0, 1, 0, q;\n\t}"
                     : "=r"(done) : "r"(bar), "r"(par) : "memory");
        if (done) return;
        if (spin == 0) start = globaltimer_ns();
        else if ((spin & 63) == 0 && globaltimer_ns() - start > 2000000000ull) {
            *(volatile int *)fail = 1;
            atomicAdd_system(timeouts, 1);
            return;
        }
    }
}

template <int DT>
__global__ void __launch_bounds__(kStreamThreads, 1) gemv_stream_kernel(float *y, const uint8_t *tiles, int ntiles, int k, VecArg x,
                                                                         StreamPlan pl, int *timeouts) {
    extern __shared__ __align__(16) unsigned char smem_stream[];
    __shared__ __align__(8) unsigned long long full[kStreamStages], empty[kStreamStages];
    __shared__ int fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bb = stream_unit_bytes(DT), nb = k / kQB;
    const size_t tb = (size_t)nb * bb;
    Prep p = carve_prep(smem_stream, k);
    unsigned char *stage0 = smem_stream + ((prep_smem(k) + 127) & ~(size_t)127);   // 16-byte aligned (bulk copy destinations)
    float2 *scratch = (float2 *)(stage0 + (size_t)kStreamStages * pl.stage_bytes);
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x), t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    const int nch = (nb + pl.U - 1) / pl.U, total = (t1 - t0 + pl.G - 1) / pl.G * nch;
    if (tid == 0) {
        fail = 0;
        for (int i = 0; i < kStreamStages; i++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&empty[i])), "r"(kStreamWarps) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();                                                       // the barriers are initialised
    // Launched as a programmatic dependent: everything above overlaps the previous kernel's tail. Unless
    // the caller declared the tiles constant (pl.early), no global memory is read before that kernel
    // has completed (its writes, x or the tiles, visible); with constant tiles the first ring of weight
    // copies starts at once and only x waits.
    if (!pl.early) asm volatile("griddepcontrol.wait;" ::: "memory");
    // The producer: chunk c of this CTA's tiles into stage c % kStreamStages, once the compute warps
    // have released that stage (from the second round of the ring on).
    auto issue = [&](int c) {
        const int st = c % kStreamStages;
        if (c >= kStreamStages) mbar_wait(smem_u32(&empty[st]), (uint32_t)(c / kStreamStages + 1) & 1u, &fail, timeouts);
        const int g0 = t0 + c / nch * pl.G, ng = min(pl.G, t1 - g0), b0 = c % nch * pl.U, nu = min(pl.U, nb - b0);
        unsigned char *buf = stage0 + (size_t)st * pl.stage_bytes;
        const uint32_t bar = smem_u32(&full[st]);
        if (lane == 0) asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)(ng * nu * bb)) : "memory");
        __syncwarp();
        for (int g = lane; g < ng; g += 32)
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                         ::"r"(smem_u32(buf + (size_t)g * pl.piece)), "l"(tiles + (size_t)(g0 + g) * tb + (size_t)b0 * bb),
                         "r"((uint32_t)(nu * bb)), "r"(bar) : "memory");
    };
    const int early = min(total, kStreamStages);                           // the first ring needs no release
    if (warp == kStreamWarps)
        for (int c = 0; c < early; c++) issue(c);                          // the weights stream in while x is loaded
    if (pl.early) asm volatile("griddepcontrol.wait;" ::: "memory");       // x may be the previous launch's output
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");        // the next launch may start its prologue
    load_prep(DT, x, k, p);                                                // every thread; ends with __syncthreads
    if (warp == kStreamWarps) {
        for (int c = early; c < total; c++) issue(c);
        return;                                                            // every chunk it started is waited for by the compute warps
    }
    const uint32_t *xw = (const uint32_t *)p.q8;
    float acc = 0.0f;
    for (int c = 0; c < total; c++) {
        const int st = c % kStreamStages, g0 = t0 + c / nch * pl.G, ng = min(pl.G, t1 - g0), cb = c % nch, b0 = cb * pl.U,
                  nu = min(pl.U, nb - b0);
        const unsigned char *buf = stage0 + (size_t)st * pl.stage_bytes;
        mbar_wait(smem_u32(&full[st]), (uint32_t)(c / kStreamStages) & 1u, &fail, timeouts);
        if (DT == DT_BF16) {
            if (tid < ng * kTile) {                                         // output (tile g, row r): its chain over the chunk's inputs
                const int g = tid >> 4, r = tid & 15;
                const uint32_t *w = (const uint32_t *)(buf + (size_t)g * pl.piece) + r;
                const float *xf = p.xf + (size_t)b0 * kQB;
                for (int q = 0; q < nu * 16; q += 8) {
                    uint32_t v[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) v[j] = w[(q + j) * kTile];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        acc = __fmaf_rn(l3m_bits_f32(v[j] << 16), xf[2 * (q + j)], acc);
                        acc = __fmaf_rn(l3m_bits_f32(v[j] & 0xFFFF0000u), xf[2 * (q + j) + 1], acc);
                    }
                }
            }
        } else {
            const int per_u = ng * 4, items = per_u * nu;
            for (int i = tid; i < items; i += 32 * kStreamWarps) {
                const int u = i / per_u, rem = i - u * per_u, g = rem >> 2, r4 = rem & 3, b = b0 + u;
                QLoad4 q;
                qload4_shared<DT>(q, smem_u32(buf + (size_t)g * pl.piece + (size_t)u * bb), r4);
                const uint4 x0 = *(const uint4 *)(xw + 8 * b), x1 = *(const uint4 *)(xw + 8 * b + 4);
                const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const float sx = p.scale[b];
                const int32_t xs = p.sum[b];
                float4 r0, r1;
                r0.x = __fmul_rn(sx, qscale4<DT>(q.d, 0)); r0.y = __int2float_rn(qdot4<DT>(q, 0, xv, xs));
                r0.z = __fmul_rn(sx, qscale4<DT>(q.d, 1)); r0.w = __int2float_rn(qdot4<DT>(q, 1, xv, xs));
                r1.x = __fmul_rn(sx, qscale4<DT>(q.d, 2)); r1.y = __int2float_rn(qdot4<DT>(q, 2, xv, xs));
                r1.z = __fmul_rn(sx, qscale4<DT>(q.d, 3)); r1.w = __int2float_rn(qdot4<DT>(q, 3, xv, xs));
                float4 *dst = (float4 *)(scratch + (size_t)b * pl.G * kTile + g * kTile + 4 * r4);
                dst[0] = r0;
                dst[1] = r1;
            }
        }
        __syncwarp();                                                       // this warp is done with the stage buffer
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[st])) : "memory");
        if (cb == nch - 1) {                                                // the wave's last blocks
            if (DT != DT_BF16) {
                asm volatile("bar.sync 1, %0;" ::"n"(32 * kStreamWarps) : "memory");   // every pair of the wave written
                if (tid < ng * kTile) {
                    const float2 *r = scratch + tid;
#pragma unroll 8
                    for (int b = 0; b < nb; b++) {
                        const float2 v = r[(size_t)b * pl.G * kTile];
                        acc = __fmaf_rn(v.x, v.y, acc);
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"n"(32 * kStreamWarps) : "memory");   // read before the next wave writes
            }
            if (tid < ng * kTile) y[(size_t)(g0 + (tid >> 4)) * kTile + (tid & 15)] = *(volatile int *)&fail ? __int_as_float(0x7FC00000) : acc;
            acc = 0.0f;
        }
    }
}

// ---- Warp-streamed exact matvec (q8_0, q4_0, mxfp4; k a multiple of 32). One CTA per SM takes a
// contiguous run of tiles [t0, t1), in waves of G tiles whose (scale product, dot) pairs fit the
// scratch. The tiles are cut into pieces of kWarpPieceBlocks 32-input blocks (one contiguous range of
// a tile); warp w takes pieces w, w + 8, ... and streams them through its own ring of kWarpStages
// shared-memory buffers: its lane 0 issues one cp.async.bulk per piece (this CTA's shared memory, no
// multicast), completing on that buffer's mbarrier, and refills the buffer as soon as the warp has
// read it. So no warp waits for another while the weights stream. Each lane computes one item per
// piece (4 rows x 1 block: the exact integer dots with dp4a) and leaves {RN(sx*d), (float)dot} in the
// wave's scratch; after one CTA barrier per wave, one thread per output runs acc = fma(RN(sx*d), dot,
// acc) over the blocks in order: the scalar kernel's rounding sequence (src/kernels_scalar.c:30-75).
constexpr int kWarpWarps = 8, kWarpThreads = 32 * kWarpWarps;
constexpr int kWarpStages = 4;
constexpr int kWarpPieceBlocks = 8;                 // 4 row groups x 8 blocks: one item per lane
constexpr size_t kWarpScratchCap = 64 * 1024;       // (scale product, dot) pairs of a wave

__host__ __device__ inline int warp_piece_bytes(int dtype) { return kWarpPieceBlocks * block_bytes(dtype); }   // a multiple of 16

size_t warp_fixed_bytes(int dtype, int k) {                            // the activation and the buffer rings
    return ((prep_smem(k) + 127) & ~(size_t)127) + (size_t)kWarpWarps * kWarpStages * warp_piece_bytes(dtype);
}
size_t smem_optin();
int stream_sms();
// The wave size for a quantised matvec of ntiles tiles of k inputs: the most tiles (at most 16, one
// output per thread, and at most one CTA's share) whose pairs fit kWarpScratchCap beside the fixed
// parts within the opt-in shared memory; 0 when the kernel does not take the shape.
int warp_plan_G(int dtype, int k, int ntiles) {
    if (dtype < DT_Q8 || k % kQB || ntiles <= 0) return 0;
    const size_t fixed = warp_fixed_bytes(dtype, k), optin = smem_optin(), per_tile = (size_t)(k / kQB) * kTile * sizeof(float2);
    if (fixed + 1024 >= optin) return 0;
    const size_t scratch = std::min(kWarpScratchCap, optin - 1024 - fixed);
    const int grid = std::min(ntiles, stream_sms()), per_cta = (ntiles + grid - 1) / grid;
    return (int)std::min<size_t>((size_t)std::min(16, per_cta), scratch / per_tile);
}

template <int DT>
__global__ void __launch_bounds__(kWarpThreads, 1) gemv_warp_kernel(float *y, const uint8_t *tiles, int ntiles, int k, VecArg x, int G, int early,
                                                                     int *timeouts) {
    extern __shared__ __align__(16) unsigned char smem_w[];
    __shared__ __align__(8) unsigned long long full[kWarpWarps][kWarpStages];
    __shared__ int fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bb = block_bytes(DT), nb = k / kQB, ppt = (nb + kWarpPieceBlocks - 1) / kWarpPieceBlocks, pbytes = warp_piece_bytes(DT);
    const size_t tb = (size_t)nb * bb;
    Prep p = carve_prep(smem_w, k);
    unsigned char *ring = smem_w + ((prep_smem(k) + 127) & ~(size_t)127);   // 16-byte aligned (bulk copy destinations)
    float2 *scratch = (float2 *)(ring + (size_t)kWarpWarps * kWarpStages * pbytes);
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x), t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    const int nt = t1 - t0, total = nt * ppt;                               // pieces of this CTA, tile-major
    if (G < 1) return;                                                     // the host never launches this (uniform)
    if (tid == 0) {
        fail = 0;
        for (int w = 0; w < kWarpWarps; w++)
            for (int i = 0; i < kWarpStages; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[w][i])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();                                                       // the barriers are initialised
    // A programmatic dependent: unless the tiles are declared constant, no global memory is read before
    // the previous kernel on the stream has completed; with constant tiles only x waits.
    if (!early) asm volatile("griddepcontrol.wait;" ::: "memory");
    // This warp's j-th piece (CTA piece warp + 8 j) into its buffer j % kWarpStages.
    auto issue = [&](int j) {
        const int i = warp + kWarpWarps * j;
        if (i >= total || lane != 0) return;
        const int tl = i / ppt, b0 = (i - tl * ppt) * kWarpPieceBlocks, nbk = min(kWarpPieceBlocks, nb - b0);
        const uint32_t bar = smem_u32(&full[warp][j % kWarpStages]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)(nbk * bb)) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(smem_u32(ring + (size_t)(warp * kWarpStages + j % kWarpStages) * pbytes)),
                     "l"(tiles + (size_t)(t0 + tl) * tb + (size_t)b0 * bb), "r"((uint32_t)(nbk * bb)), "r"(bar) : "memory");
    };
    for (int j = 0; j < kWarpStages; j++) issue(j);                        // the weights stream in while x is loaded
    if (early) asm volatile("griddepcontrol.wait;" ::: "memory");          // x may be the previous launch's output
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    load_prep(DT, x, k, p);                                                // every thread; ends with __syncthreads
    const uint32_t *xw = (const uint32_t *)p.q8;
    const int r4 = lane & 3, u = lane >> 2;                                 // this lane's item in a piece: rows 4 r4.., block u
    int j = 0;
    for (int tw0 = 0; tw0 < nt; tw0 += G) {
        const int tw1 = min(nt, tw0 + G), n_out = (tw1 - tw0) * kTile;
        for (;; j++) {                                                      // this warp's pieces of the wave
            const int i = warp + kWarpWarps * j;
            if (i >= total || i / ppt >= tw1) break;
            const int st = j % kWarpStages, tl = i / ppt, b0 = (i - tl * ppt) * kWarpPieceBlocks, nbk = min(kWarpPieceBlocks, nb - b0);
            mbar_wait(smem_u32(&full[warp][st]), (uint32_t)(j / kWarpStages) & 1u, &fail, timeouts);
            if (u < nbk) {
                const int b = b0 + u;
                QLoad4 q;
                qload4_shared<DT>(q, smem_u32(ring + (size_t)(warp * kWarpStages + st) * pbytes + (size_t)u * bb), r4);
                const uint4 x0 = *(const uint4 *)(xw + 8 * b), x1 = *(const uint4 *)(xw + 8 * b + 4);
                const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const float sx = p.scale[b];
                const int32_t xs = p.sum[b];
                float4 r0, r1;
                r0.x = __fmul_rn(sx, qscale4<DT>(q.d, 0)); r0.y = __int2float_rn(qdot4<DT>(q, 0, xv, xs));
                r0.z = __fmul_rn(sx, qscale4<DT>(q.d, 1)); r0.w = __int2float_rn(qdot4<DT>(q, 1, xv, xs));
                r1.x = __fmul_rn(sx, qscale4<DT>(q.d, 2)); r1.y = __int2float_rn(qdot4<DT>(q, 2, xv, xs));
                r1.z = __fmul_rn(sx, qscale4<DT>(q.d, 3)); r1.w = __int2float_rn(qdot4<DT>(q, 3, xv, xs));
                float4 *dst = (float4 *)(scratch + (size_t)b * n_out + (tl - tw0) * kTile + 4 * r4);
                dst[0] = r0;
                dst[1] = r1;
            }
            __syncwarp();                                                   // every lane has read the buffer
            issue(j + kWarpStages);                                         // refill it (possibly with the next wave's piece)
        }
        __syncthreads();                                                    // every pair of the wave written
        if (tid < n_out) {
            const float2 *r = scratch + tid;
            float acc = 0.0f;
#pragma unroll 8
            for (int b = 0; b < nb; b++) {
                const float2 v = r[(size_t)b * n_out];
                acc = __fmaf_rn(v.x, v.y, acc);
            }
            y[(size_t)(t0 + tw0) * kTile + tid] = *(volatile int *)&fail ? __int_as_float(0x7FC00000) : acc;
        }
        __syncthreads();                                                    // read before the next wave writes
    }
}

// Fast f32/bf16: one warp per tile; each half warp walks alternate 16-input chunks for its 16 outputs.
__global__ void __launch_bounds__(kThreads) gemv_fast_kernel(int dtype, float *y, const uint8_t *tiles, int ntiles, int k, VecArg x) {
    const int lane = threadIdx.x & 31, warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nwarps = gridDim.x * (blockDim.x >> 5), c = lane & 15, half = lane >> 4;
    const size_t tb = tile_bytes(dtype, k);
    for (int t = warp; t < ntiles; t += nwarps) {
        const uint8_t *tile = tiles + (size_t)t * tb;
        float a0 = 0.0f, a1 = 0.0f;
        if (dtype == DT_BF16) {
            const uint32_t *w = (const uint32_t *)tile + c;
            for (int q = half; q < k / 2; q += 2) {
                const uint32_t v = ld_nc_u32(w + (size_t)q * kTile);
                a0 = fmaf(l3m_bits_f32(v << 16), l3m_bf16_to_f32(x.bf16[2 * q]), a0);
                a1 = fmaf(l3m_bits_f32(v & 0xFFFF0000u), l3m_bf16_to_f32(x.bf16[2 * q + 1]), a1);
            }
        } else {
            const float *w = (const float *)tile + c;
            for (int i = half; i < k; i += 2) a0 = fmaf(__ldg(w + (size_t)i * kTile), x.f32[i], a0);
        }
        float acc = a0 + a1;
        acc += __shfl_xor_sync(0xffffffffu, acc, 16);
        if (!half) y[(size_t)t * kTile + c] = acc;
    }
}

// Exact integer block dots, one warp (q8) or half warp (q4, mxfp4) per (tile, block).
template <int DT>
__device__ void block_dots_items(int32_t *dots, const uint8_t *tiles, int ntiles, int k, const VecArg &x) {
    const int nb = k / kQB, bb = block_bytes(DT);
    const size_t tb = (size_t)nb * bb;
    const long long n = (long long)ntiles * kTile, items = n * nb;
    const uint32_t *xw = (const uint32_t *)x.q8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < items; i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / n);
        const long long o = i - (long long)b * n;
        QLoad q;
        qload<DT>(q, tiles + (size_t)(o >> 4) * tb + (size_t)b * bb, (int)(o & 15));
        dots[o * nb + b] = qdot<DT>(q, xw + 8 * b, x.sum[b]);
    }
}

// Exact integer block dots: one thread per (output, block).
__global__ void block_dots_kernel(int dtype, int32_t *dots, const uint8_t *tiles, int ntiles, int k, VecArg x) {
    if (dtype == DT_Q8) block_dots_items<DT_Q8>(dots, tiles, ntiles, k, x);
    else if (dtype == DT_Q4) block_dots_items<DT_Q4>(dots, tiles, ntiles, k, x);
    else block_dots_items<DT_MX>(dots, tiles, ntiles, k, x);
}

// Unpack: one thread per (output, block).
__global__ void unpack_kernel(int dtype, int8_t *q, float *d, const uint8_t *tiles, int ntiles, int k) {
    const int nb = k / kQB, bb = block_bytes(dtype);
    const size_t tb = (size_t)nb * bb;
    const long long n = (long long)ntiles * kTile * nb;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < n; id += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(id % nb);
        const long long o = id / nb;
        const int t = (int)(o / kTile), c = (int)(o % kTile);
        const uint8_t *blk = tiles + (size_t)t * tb + (size_t)b * bb;
        int8_t *qo = q + o * k + b * kQB;
        if (dtype == DT_Q8) {
            d[o * nb + b] = l3m_f16_to_f32(ld_nc_u16(blk + 2 * c));
            for (int i = 0; i < kQB; i++) qo[i] = (int8_t)(ld_nc_u8(blk + 32 + ((i / 4) * kTile + c) * 4 + i % 4) - 128);
        } else {
            const int sb = dtype == DT_MX ? 16 : 32;
            d[o * nb + b] = dtype == DT_MX ? l3m_e8m0_half(ld_nc_u8(blk + c)) : l3m_f16_to_f32(ld_nc_u16(blk + 2 * c));
            for (int i = 0; i < kQB; i++) {
                const int g = i / 8, j = i % 8;
                const uint8_t byte = ld_nc_u8(blk + sb + (g * kTile + c) * 4 + (j & 3));
                const int nib = j < 4 ? (byte & 15) : (byte >> 4);
                qo[i] = (int8_t)(dtype == DT_MX ? l3m_mxfp4_value(nib) : nib - 8);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) prepare_kernel(int dtype, const float *x, int n, int8_t *q8, float *scale, int32_t *sum, uint16_t *bf16) {
    const int tid = threadIdx.x + blockIdx.x * blockDim.x, nth = blockDim.x * gridDim.x;
    if (dtype == DT_BF16) {
        for (int i = tid; i < n; i += nth) bf16[i] = l3m_f32_to_bf16(x[i]);
        return;
    }
    const int lane = threadIdx.x & 31, gw = tid >> 5, nw = nth >> 5;
    for (int b = gw; b < n / kQB; b += nw) {
        const float v = x[b * kQB + lane], a = fabsf(v);
        const float amax = warp_max_f32(a > 0.0f ? a : 0.0f);
        const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        const int8_t q = (int8_t)__float2int_rn(__fmul_rn(v, inv));
        q8[b * kQB + lane] = q;
        const int s = warp_sum_i32((int)q);
        if (lane == 0) { scale[b] = __fdiv_rn(amax, 127.0f); sum[b] = s; }
    }
}

__global__ void __launch_bounds__(kThreads) attend_kernel(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int hd,
                                                          int stride, const uint32_t *etab) {
    extern __shared__ __align__(16) unsigned char smem[];
    float *qs = (float *)smem, *o = qs + hd, *red = o + hd, *scores = red + 64;
    uint16_t *kcur = (uint16_t *)(scores + ((pos + 4) & ~3)), *vcur = kcur + hd, *kvbuf = vcur + hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        qs[i] = q[i];
        kcur[i] = k[(size_t)pos * stride + i];
        vcur[i] = v[(size_t)pos * stride + i];
    }
    __syncthreads();
    attend_exact<false>(qs, k, v, stride, stride, kcur, vcur, pos, hd, scores, o, red, etab, kvbuf, nullptr, kAttnChunk, false);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) out[i] = o[i];
}

VecArg vec_arg(const l3m_vec *x) { return VecArg{x->f32, x->bf16, x->q8, x->scale, x->sum}; }

// One warp-streamed matvec launch, a programmatic dependent launch like launch_stream's.
template <class K>
cudaError_t launch_warp(K kernel, int grid, size_t smem, cudaStream_t s, float *y, const uint8_t *t, int ntiles, int k, VecArg x, int G,
                        int early, int *tmo) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kWarpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, y, t, ntiles, k, x, G, early, tmo);
}

// One streamed-matvec launch as a programmatic dependent launch: the kernel's prologue (shared-memory
// barriers) may run while the previous work on the stream finishes; the kernel waits for that work
// (griddepcontrol.wait) before it reads any global memory.
template <class K>
cudaError_t launch_stream(K kernel, int grid, size_t smem, cudaStream_t s, float *y, const uint8_t *t, int ntiles, int k, VecArg x,
                          StreamPlan pl, int *tmo) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, y, t, ntiles, k, x, pl, tmo);
}

// The kernels read tiles with 16-byte (and 4-byte) loads and x, y as 4-byte words: a misaligned
// pointer would fault the caller's context, so it is refused before anything launches.
bool misaligned_args(int dtype, const void *y, const void *tiles, const l3m_vec *x) {
    uintptr_t w = (uintptr_t)y | (uintptr_t)tiles;
    if (dtype == DT_F32) w |= (uintptr_t)x->f32;
    else if (dtype == DT_BF16) w |= (uintptr_t)x->bf16 & 1;
    else w |= (uintptr_t)x->q8 | (uintptr_t)x->scale | (uintptr_t)x->sum | ((uintptr_t)tiles & 15);
    return (w & 3) != 0 || (dtype >= DT_Q8 && ((uintptr_t)tiles & 15) != 0);
}

// The streamed kernel's count of waits that gave up, in host-mapped memory (one counter for every
// device: the host pointer is the device pointer under unified addressing). A count that changed
// since the last call means an earlier launch wrote NaN outputs: this call reports it and fails.
int stream_timeouts(int **dev_ptr) {
    static std::mutex mu;
    static int *host = nullptr, seen = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!host) {
        cudaError_t e = cudaHostAlloc((void **)&host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) { host = nullptr; return fail(e, "l3m_gemv_dev: host-mapped timeout counter"); }
        *host = 0;
    }
    const int now = *(volatile int *)host;
    if (now != seen) {
        snprintf(g_err, sizeof g_err, "l3m_gemv_dev: %d weight-copy wait(s) of an earlier launch gave up; its y holds NaN", now - seen);
        seen = now;
        return -1;
    }
    *dev_ptr = host;
    return 0;
}

int stream_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

size_t smem_optin() {
    static int v = 0;
    if (!v) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    return (size_t)v;
}

int grid_for(int ntiles) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    int g = 2 * sms;
    return ntiles < g ? (ntiles > 0 ? ntiles : 1) : g;
}

}  // namespace

// ---- expf exception list on the device (shared with the decode engine)
#include "expf_exceptions.inc"

extern "C" int l3m_expf_table(const uint32_t **table) {
    static std::mutex mu;
    static const uint32_t *d_table[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return fail_msg("no CUDA device");
    std::lock_guard<std::mutex> lock(mu);
    if (L3M_EXPF_LIST_N == 0) {                                      // the C library follows the method: nothing to look up
        *table = nullptr;
        return 0;
    }
    if (!d_table[dev]) {
        std::vector<uint32_t> h(L3M_EXPF_SLOTS);
        if (l3m_expf_hash_build(l3m_expf_list_host, L3M_EXPF_LIST_N, h.data())) return fail_msg("expf exception set does not fit its table");
        uint32_t *t = nullptr;
        cudaError_t e = cudaMalloc(&t, h.size() * sizeof(uint32_t));
        if (e == cudaSuccess) e = cudaMemcpy(t, h.data(), h.size() * sizeof(uint32_t), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail(e, "expf table");
        d_table[dev] = t;
    }
    *table = d_table[dev];
    return 0;
}

// The latency of one step of a dependent fp32 chain (acc = fma(acc, a, b), operands in registers),
// timed by the SM's cycle counter: the per-step cost of the sequential sums and fma chains that bound
// the decode. The read of acc before the second stamp waits for the chain's last step.
__device__ long long g_chain_cycles;
__device__ float g_chain_sink;
__global__ void chain_kernel(int steps, float a, float b) {
    float acc = 0.0f;
    const long long t0 = clock64();
#pragma unroll 8
    for (int i = 0; i < steps; i++) acc = __fmaf_rn(acc, a, b);
    if (__float_as_uint(acc) == 0x7FC00001u) g_chain_sink = acc;
    const long long t1 = clock64();
    if (threadIdx.x == 0) {
        g_chain_cycles = t1 - t0;
        g_chain_sink = acc;
    }
}

__global__ void expf_kernel(const float *__restrict__ x, float *__restrict__ y, int n, const uint32_t *etab) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = l3m_expf_exact(x[i], etab);
}

// Error text for the other entry-point files of this library (not exported).
extern "C" int l3m_error_msg(const char *msg) { return fail_msg(msg); }
extern "C" int l3m_error_cuda(int e, const char *what) { return fail((cudaError_t)e, what); }

extern "C" {

L3M_API const char *l3m_cuda_error(void) { return g_err; }

L3M_API int l3m_chain_cycles_dev(int steps, double *cycles_per_step) {
    if (steps < 64 || steps > (1 << 24) || !cycles_per_step) return fail_msg("l3m_chain_cycles_dev: bad arguments (steps in [64, 2^24])");
    long long cyc = 0;
    for (int run = 0; run < 2; run++) {                               // the second run, warm
        chain_kernel<<<1, 32>>>(steps, 0.999f, 0.001f);
        cudaError_t e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&cyc, g_chain_cycles, sizeof cyc);
        if (e != cudaSuccess) return fail(e, "l3m_chain_cycles_dev");
    }
    *cycles_per_step = (double)cyc / steps;
    return 0;
}

L3M_API int l3m_expf_dev(const float *x, float *y, int n, void *stream) {
    if (n < 0 || (n > 0 && (!x || !y))) return fail_msg("l3m_expf_dev: bad arguments");
    const uint32_t *etab;
    if (l3m_expf_table(&etab)) return -1;
    if (n == 0) return 0;
    const int blocks = std::min((n + 255) / 256, 148 * 8);
    expf_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(x, y, n, etab);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_expf_dev");
}

L3M_API int l3m_gemv_dev(int exact, int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream) {
    if (dtype < 0 || dtype >= L3M_DT_COUNT || ntiles < 0 || k <= 0) return fail_msg("l3m_gemv_dev: bad arguments");
    if (dtype >= DT_Q8 && k % kQB) return fail_msg("l3m_gemv_dev: quantised k must be a multiple of 32");
    if (dtype == DT_BF16 && k % 2) return fail_msg("l3m_gemv_dev: bf16 k must be even");
    if (ntiles == 0) return 0;
    if (!y || !tiles || !x) return fail_msg("l3m_gemv_dev: y, tiles and x are required");
    if (misaligned_args(dtype, y, tiles, x)) return fail_msg("l3m_gemv_dev: misaligned pointer (y, f32/q8/scale/sum and bf16/f32 tiles 4-byte, quantised tiles 16-byte, bf16 x 2-byte)");
    int *tmo = nullptr;
    if (stream_timeouts(&tmo)) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    static const bool stream_off = getenv("L3M_GEMV_STREAM") && !strcmp(getenv("L3M_GEMV_STREAM"), "0");
    if (!(exact & 1) && dtype <= DT_BF16) {
        gemv_fast_kernel<<<grid_for((ntiles + 15) / 16), kThreads, 0, s>>>(dtype, y, (const uint8_t *)tiles, ntiles, k, vec_arg(x));
    } else if (const int G = warp_plan_G(dtype, k, ntiles); !stream_off && G > 0 && ((uintptr_t)tiles & 15) == 0) {
        const int grid = std::min(ntiles, stream_sms());
        const size_t smem = warp_fixed_bytes(dtype, k) + (size_t)G * (k / kQB) * kTile * sizeof(float2);
        const int early = (exact & kConstTiles) ? 1 : 0;
        const uint8_t *t = (const uint8_t *)tiles;
        cudaError_t e = cudaSuccess;
        switch (dtype) {
        case DT_Q8: e = launch_warp(gemv_warp_kernel<DT_Q8>, grid, smem, s, y, t, ntiles, k, vec_arg(x), G, early, tmo); break;
        case DT_Q4: e = launch_warp(gemv_warp_kernel<DT_Q4>, grid, smem, s, y, t, ntiles, k, vec_arg(x), G, early, tmo); break;
        default: e = launch_warp(gemv_warp_kernel<DT_MX>, grid, smem, s, y, t, ntiles, k, vec_arg(x), G, early, tmo); break;
        }
        if (e != cudaSuccess) return fail(e, "l3m_gemv_dev");
    } else if (!stream_off && dtype >= DT_BF16 && k % kQB == 0 && ((uintptr_t)tiles & 15) == 0 && stream_plan(dtype, k, 16).G &&
               stream_smem(k, stream_plan(dtype, k, 16)) + 1024 <= smem_optin()) {
        const int grid = std::min(ntiles, stream_sms());
        StreamPlan pl = stream_plan(dtype, k, (ntiles + grid - 1) / grid);
        pl.early = (exact & kConstTiles) ? 1 : 0;
        const size_t smem = stream_smem(k, pl);
        cudaError_t e = cudaSuccess;
        const uint8_t *t = (const uint8_t *)tiles;
        switch (dtype) {
        case DT_BF16: e = launch_stream(gemv_stream_kernel<DT_BF16>, grid, smem, s, y, t, ntiles, k, vec_arg(x), pl, tmo); break;
        case DT_Q8: e = launch_stream(gemv_stream_kernel<DT_Q8>, grid, smem, s, y, t, ntiles, k, vec_arg(x), pl, tmo); break;
        case DT_Q4: e = launch_stream(gemv_stream_kernel<DT_Q4>, grid, smem, s, y, t, ntiles, k, vec_arg(x), pl, tmo); break;
        default: e = launch_stream(gemv_stream_kernel<DT_MX>, grid, smem, s, y, t, ntiles, k, vec_arg(x), pl, tmo); break;
        }
        if (e != cudaSuccess) return fail(e, "l3m_gemv_dev");
    } else {
        const int per_cta = (ntiles + grid_for(ntiles) - 1) / grid_for(ntiles);
        size_t smem = prep_smem(k) + (size_t)kScratchPairs * sizeof(float2) + (size_t)per_cta * kTile * 4;
        if (dtype >= DT_Q8 && (size_t)(k / kQB) * kTile > (size_t)kScratchPairs) return fail_msg("l3m_gemv_dev: k too large");
        cudaError_t e = cudaFuncSetAttribute(gemv_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail(e, "l3m_gemv_dev");
        gemv_exact_kernel<<<grid_for(ntiles), kThreads, smem, s>>>(dtype, y, (const uint8_t *)tiles, ntiles, k, vec_arg(x));
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_gemv_dev");
}

L3M_API int l3m_vec_prepare_dev(int dtype, l3m_vec *out, const float *x, int n, void *scratch, void *stream) {
    if (dtype < 0 || dtype >= L3M_DT_COUNT || n <= 0) return fail_msg("l3m_vec_prepare_dev: bad arguments (dtype, n > 0)");
    if (dtype >= DT_Q8 && n % kQB) return fail_msg("l3m_vec_prepare_dev: n must be a multiple of 32");
    if (!out || !x || (dtype != DT_F32 && !scratch)) return fail_msg("l3m_vec_prepare_dev: out, x and (but for f32) scratch are required");
    memset(out, 0, sizeof *out);
    out->f32 = x;
    if (dtype == DT_F32) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    int8_t *q = (int8_t *)scratch;
    float *scale = (float *)(q + n);
    int32_t *sum = (int32_t *)(scale + n / kQB);
    int grid = (n + kThreads - 1) / kThreads;
    if (dtype == DT_BF16) {
        prepare_kernel<<<grid, kThreads, 0, s>>>(dtype, x, n, nullptr, nullptr, nullptr, (uint16_t *)scratch);
        out->bf16 = (const uint16_t *)scratch;
    } else {
        prepare_kernel<<<grid, kThreads, 0, s>>>(dtype, x, n, q, scale, sum, nullptr);
        out->q8 = q; out->scale = scale; out->sum = sum;
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_vec_prepare_dev");
}

L3M_API int l3m_block_dots_dev(int dtype, int32_t *dots, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream) {
    if (dtype < DT_Q8 || dtype > DT_MX || k <= 0 || k % kQB || ntiles < 0)
        return fail_msg("l3m_block_dots_dev: quantised dtypes, k a positive multiple of 32, ntiles >= 0");
    if (ntiles == 0) return 0;
    if (!dots || !tiles || !x || !x->q8 || !x->sum) return fail_msg("l3m_block_dots_dev: dots, tiles and a prepared x are required");
    block_dots_kernel<<<grid_for(ntiles), 256, 0, (cudaStream_t)stream>>>(dtype, dots, (const uint8_t *)tiles, ntiles, k, vec_arg(x));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_block_dots_dev");
}

L3M_API int l3m_unpack_dev(int dtype, int8_t *q, float *d, const void *tiles, int ntiles, int k, void *stream) {
    if (dtype < DT_Q8 || dtype > DT_MX || k <= 0 || k % kQB || ntiles < 0)
        return fail_msg("l3m_unpack_dev: quantised dtypes, k a positive multiple of 32, ntiles >= 0");
    if (ntiles == 0) return 0;
    if (!q || !d || !tiles) return fail_msg("l3m_unpack_dev: q, d and tiles are required");
    unpack_kernel<<<grid_for(ntiles), 256, 0, (cudaStream_t)stream>>>(dtype, q, d, (const uint8_t *)tiles, ntiles, k);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_unpack_dev");
}

L3M_API int l3m_attend_dev(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int head_dim, int stride, void *stream) {
    if (head_dim % 8 || head_dim <= 0 || pos < 0 || stride < head_dim) return fail_msg("l3m_attend_dev: bad arguments");
    if (!out || !q || !k || !v) return fail_msg("l3m_attend_dev: out, q, k and v are required");
    const uint32_t *etab;
    if (l3m_expf_table(&etab)) return -1;
    size_t smem = (size_t)head_dim * 8 + 64 * 4 + (size_t)((pos + 4) & ~3) * 4 + (size_t)head_dim * 4 + 16 +
                  (size_t)kAttnChunk * (head_dim + 8) * 2;
    cudaError_t e = cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(e, "l3m_attend_dev");
    attend_kernel<<<1, kThreads, smem, (cudaStream_t)stream>>>(out, q, k, v, pos, head_dim, stride, etab);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail(e, "l3m_attend_dev");
}

}  // extern "C"
