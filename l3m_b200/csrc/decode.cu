// The decode kernel: one launch runs a whole l3m_generate call (prompt feed and greedy sampling) on
// one GPU: one thread-block cluster of kClusterCtas CTAs (cluster 0) runs the layers, and the other
// clusters of the launch (the helpers, as many as the GPU holds) run the head. Replaces the
// reference's pinned thread pool and its four barriers per layer (src/engine.c:230-281,
// src/pool.c:111-123).
//
// Every CTA keeps the residual x in its shared memory. Each matrix is split into contiguous runs of
// 16-row tiles over the CTAs (the reference's split over ranks, src/engine.c:88-91). A CTA writes
// its slice of every produced vector straight into the shared memory of all CTAs of the cluster
// (distributed shared memory) with st.async, each store completing its bytes on the receiver's
// mbarrier for that exchange, so an exchange needs no global-memory round trip and no cluster
// barrier (when some CTA has no qkv rows, hardware cluster barriers order the exchanges instead).
// Per layer:
//   Q  qkv CTAs:  rmsnorm, their tiles of the q/k/v rows                   -> qkv      exchange 1
//   A  head CTAs: RoPE, KV row, attention (K/V copies started during Q)   -> attn     exchange 2
//   B  wo CTAs:   matvec                                                  -> proj     exchange 3
//   C  all:       x += proj; ffn CTAs: rmsnorm, up and gate, SiLU gate    -> h        exchange 4
//   D  down CTAs: matvec                                                  -> down     exchange 5
//   all:          x += down
// After the last prompt position each position ends with the head matvec (logits kept for
// l3m_logits) on the helper clusters (on every CTA in cold mode), a per-CTA argmax posted as one
// slot word, and the same global argmax in every CTA of cluster 0, in CTA order. Each exchanged
// vector has one buffer: its next write comes after every reader has finished with it. The weight
// tiles of the next matvec phase are copied into shared memory by the tensor memory accelerator
// (bulk copies, this CTA's own memory) where no exchange is in flight; each layer's norm weights and
// RoPE row are copied into shared memory while the previous layer runs.
//
// Waits. Cluster barriers are reached the same number of times by every CTA of the cluster. Every
// other wait (an exchange's mbarrier, a weight copy's mbarrier, the head's x and slot words in
// global memory) polls with a time limit; a wait that gives up records an error code and where it
// was (CTA, position, layer, which wait) in the abort word, and every later wait of the launch stops
// as soon as it sees that word set, so the launch ends at the next sampled position instead of
// running every remaining wait to its limit. At entry every CTA checks that the launch has the shape
// this code assumes (kClusterCtas CTAs per cluster, whole clusters, the grid of the arguments) and
// ends at once with kErrShape otherwise, before any distributed-shared-memory access.
#include <algorithm>
#include <cstdio>
#include <cooperative_groups.h>
#include "ops.cuh"
#include "decode.cuh"
#include "../../include/l3m_kernels.h"

namespace cg = cooperative_groups;

namespace l3m {

struct Smem {
    float *x, *xb, *tmp, *y, *scores, *att, *red, *wa, *wf, *wh, *wab, *wfb, *whb;
    float *xq, *xa, *xp, *xh, *xd, *xt;
    float2 *rope;
    uint16_t *kcur, *vcur, *kvbuf, *vtbuf;
    float2 *scratch;
    uint8_t *w;                          // weight staging area
    unsigned long long *wbar;            // its mbarrier
    unsigned long long *xbar;            // exchanges 1-5 (async_x)
    Prep prep;
    Prep pa, ph;                         // q8 exchanges: the activations of wo and down as received
};

__device__ __forceinline__ Smem carve(unsigned char *base, const DecodeArgs &a) {
    Smem s;
    s.x = (float *)(base + a.sm_x);
    s.xb = (float *)(base + a.sm_xb);
    s.tmp = (float *)(base + a.sm_tmp);
    s.y = (float *)(base + a.sm_y);
    s.scores = (float *)(base + a.sm_scores);
    s.att = (float *)(base + a.sm_att);
    s.red = (float *)(base + a.sm_red);
    s.wa = (float *)(base + a.sm_wa);
    s.wf = (float *)(base + a.sm_wf);
    s.wh = (float *)(base + a.sm_wh);
    s.wab = (float *)(base + a.sm_wab);
    s.wfb = (float *)(base + a.sm_wfb);
    s.whb = (float *)(base + a.sm_whb);
    s.xq = (float *)(base + a.sm_xq);
    s.xa = (float *)(base + a.sm_xa);
    s.xp = (float *)(base + a.sm_xp);
    s.xh = (float *)(base + a.sm_xh);
    s.xd = (float *)(base + a.sm_xd);
    s.xt = (float *)(base + a.sm_xt);
    s.rope = (float2 *)(base + a.sm_rope);
    s.kcur = (uint16_t *)(base + a.sm_kv);
    s.vcur = s.kcur + a.hd;
    s.kvbuf = (uint16_t *)(base + a.sm_kvbuf);
    s.vtbuf = (uint16_t *)(base + a.sm_vt);
    s.scratch = (float2 *)(base + a.sm_scratch);
    s.w = base + (blockIdx.x >= kClusterCtas ? a.sm_w_head : a.sm_w);
    s.wbar = (unsigned long long *)(base + a.sm_wbar);
    s.xbar = (unsigned long long *)(base + a.sm_xbar);
    s.prep.q8 = (int8_t *)(base + a.sm_q8);
    s.prep.scale = (float *)(base + a.sm_scale);
    s.prep.sum = (int32_t *)(base + a.sm_sum);
    s.prep.xf = (float *)(base + a.sm_xf);
    s.pa = Prep{(int8_t *)(base + a.sm_pa_q8), (float *)(base + a.sm_pa_scale), (int32_t *)(base + a.sm_pa_sum), (float *)(base + a.sm_xa)};
    s.ph = Prep{(int8_t *)(base + a.sm_ph_q8), (float *)(base + a.sm_ph_scale), (int32_t *)(base + a.sm_ph_sum), (float *)(base + a.sm_xh)};
    return s;
}

// Every thread of every CTA of the cluster: writes before it (shared, distributed shared and global
// memory) are visible to every thread of the cluster after it.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// src[0, n) (this CTA's slice, shared memory) to dst[g0, g0 + n) in the shared memory of every CTA of
// the cluster, this one included. Visible to the readers after the next cluster_sync.
__device__ __noinline__ void scatter(const float *src, float *dst, int g0, int n) {
    cg::cluster_group cl = cg::this_cluster();
    const int tid = threadIdx.x, nth = blockDim.x, nr = (int)cl.num_blocks();
    if (((g0 | n) & 3) == 0) {
        const int n4 = n >> 2;
        #pragma unroll 1
        for (int e = tid; e < n4 * nr; e += nth) {
            const int r = e % nr, j = e / nr;
            float4 *d = (float4 *)cl.map_shared_rank(dst + g0, (unsigned)r);
            d[j] = ((const float4 *)src)[j];
        }
    } else {
        #pragma unroll 1
        for (int e = tid; e < n * nr; e += nth) {
            const int r = e % nr, j = e / nr;
            cl.map_shared_rank(dst + g0, (unsigned)r)[j] = src[j];
        }
    }
}

// Diagnostics: thread 0 of the traced CTAs stamps its SM cycle counter (clock64: a few cycles to
// read, unlike the global timer) per (position, layer, event).
// The same with st.async: each 16- (or 4-) byte store completes its bytes on the receiving CTA's
// mbarrier bar (this CTA's address of it, mapped per rank), so the receivers wait for their bytes
// instead of a cluster barrier, and the sender does not wait for its stores to land.
template <bool RB>
__device__ __forceinline__ float round_bf16(float v) { return RB ? l3m_bf16_to_f32(l3m_f32_to_bf16(v)) : v; }
// RB: each value rounded to bf16 first (the bf16 prepare's rounding); one instance each.
template <bool RB = false>
__device__ __noinline__ void scatter_tx(const float *src, float *dst, int g0, int n, unsigned long long *bar) {
    const int tid = threadIdx.x, nth = blockDim.x;
    const uint32_t ld = (uint32_t)__cvta_generic_to_shared(dst + g0), lb = (uint32_t)__cvta_generic_to_shared(bar);
    if (((g0 | n) & 3) == 0) {
        const int n4 = n >> 2;
        #pragma unroll 1
        for (int e = tid; e < n4 * kClusterCtas; e += nth) {
            const int r = e % kClusterCtas, j = e / kClusterCtas;
            uint32_t ra, rbar;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(ld + 16 * j), "r"(r));
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(lb), "r"(r));
            const float4 v = ((const float4 *)src)[j];
            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
                         ::"r"(ra), "f"(round_bf16<RB>(v.x)), "f"(round_bf16<RB>(v.y)), "f"(round_bf16<RB>(v.z)), "f"(round_bf16<RB>(v.w)),
                         "r"(rbar) : "memory");
        }
    } else {
        #pragma unroll 1
        for (int e = tid; e < n * kClusterCtas; e += nth) {
            const int r = e % kClusterCtas, j = e / kClusterCtas;
            uint32_t ra, rbar;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(ld + 4 * j), "r"(r));
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(lb), "r"(r));
            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];"
                         ::"r"(ra), "r"(__float_as_uint(round_bf16<RB>(src[j]))), "r"(rbar) : "memory");
        }
    }
}

// Only the kernel's TRACE instances carry the stamps (the others have no code for them at all).
template <bool TRACE>
__device__ __forceinline__ void trace(const DecodeArgs &a, int slot, int pos, int l, int ev) {
    if constexpr (TRACE) {
        if (slot >= 0 && threadIdx.x == 0)
            a.trace[(((size_t)slot * a.ctx + pos) * (a.n_layers + 1) + l) * kTraceEvents + ev] = (unsigned long long)clock64();
    }
}

// This CTA's share of the expf exception table into L2 with an evict-last policy (one thread; the
// table's size is a multiple of 16 bytes per CTA share rounding, and its base 256-byte aligned).
__device__ __noinline__ void prefetch_expf_table(const uint32_t *table, int cta, int ncta) {
    const uint32_t units = L3M_EXPF_SLOTS * 4 / 16, u0 = (uint32_t)((uint64_t)units * cta / ncta), u1 = (uint32_t)((uint64_t)units * (cta + 1) / ncta);
    if (u1 <= u0) return;
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"((const char *)table + 16ull * u0), "r"(16 * (u1 - u0)), "l"(pol)
                 : "memory");
}

// Pull a CTA's weight tiles into L2 ahead of use (cp.async.bulk.prefetch: no registers, no
// completion to wait for). Every tile range is 16-byte aligned and a multiple of 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    for (size_t o = 0; o < bytes; o += (1u << 20)) {
        const uint32_t n = (uint32_t)min(bytes - o, (size_t)1 << 20);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((const char *)p + o), "r"(n) : "memory");
    }
}

// Issued by thread 32 (warp 1), which is idle while warp 0 runs the serial part of the rmsnorm that
// follows: a bulk instruction can hold its thread while the copy engine takes earlier requests.
constexpr int kPrefetchThread = 32;
__device__ void prefetch_layer(const DecodeArgs &a, const LayerDev &L, const Role &r) {
    if (threadIdx.x != kPrefetchThread) return;
    const size_t tq = tile_bytes(L.dt_qkv, a.dim), to = tile_bytes(L.dt_wo, a.dim), tu = tile_bytes(L.dt_up, a.dim),
                 tg = tile_bytes(L.dt_gate, a.dim), td = tile_bytes(L.dt_down, a.ffn);
    if (r.qkv0 < r.qkv1) prefetch_l2(L.qkv + r.qkv0 * tq, (size_t)(r.qkv1 - r.qkv0) * tq);
    if (r.wo0 < r.wo1) prefetch_l2(L.wo + r.wo0 * to, (size_t)(r.wo1 - r.wo0) * to);
    if (r.ffn0 < r.ffn1) {
        if (!L.gate) prefetch_l2(L.up + 2 * r.ffn0 * tu, (size_t)2 * (r.ffn1 - r.ffn0) * tu);
        else {
            prefetch_l2(L.up + r.ffn0 * tu, (size_t)(r.ffn1 - r.ffn0) * tu);
            prefetch_l2(L.gate + r.ffn0 * tg, (size_t)(r.ffn1 - r.ffn0) * tg);
        }
    }
    if (r.dn0 < r.dn1) prefetch_l2(L.down + r.dn0 * td, (size_t)(r.dn1 - r.dn0) * td);
}

// The norm weights of layer L and the RoPE row of position pos, into shared memory (asynchronous;
// the top of the next layer waits for them). GPT2: the LayerNorm biases too (GPT-2 family).
template <bool GPT2>
__device__ __noinline__ void stage_vectors(const DecodeArgs &a, const LayerDev &L, const Role &role, const Smem &s, int pos) {
    if (role.qkv0 < role.qkv1) {
        stage_f32(s.wa, L.attn_norm, a.dim);
        if (GPT2 && a.layernorm) stage_f32(s.wab, L.attn_norm_b, a.dim);
    }
    if (role.ffn0 < role.ffn1) {
        stage_f32(s.wf, L.ffn_norm, a.dim);
        if (GPT2 && a.layernorm) stage_f32(s.wfb, L.ffn_norm_b, a.dim);
    }
    if (role.head0 >= 0 && a.rope && pos < a.ctx) stage_f32((float *)s.rope, (const float *)(a.rope + (size_t)pos * (a.hd / 2)), a.hd);
    cp_async_commit();
}

// ---- Weight staging. A CTA's quantised tiles for its next matvec phase are copied into shared
// memory by the tensor memory accelerator (cp.async.bulk: one thread issues, no registers held,
// completion counted in bytes on one mbarrier) while the current phase, its barrier and the next
// norm run; the matvec then reads shared memory. One copy is outstanding at a time: the phase that
// consumes it waits for it, and the next copy is issued only after that phase's last read.

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void stage_init(const Smem &s) {
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(s.wbar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
}

// One thread: one bulk copy of bytes (a multiple of 16, at most the staging area) from src to the
// shared address dst, completing on the mbarrier bar. cold: with an L2 evict-first policy.
__device__ __noinline__ void bulk_copy(uint32_t dst, const uint8_t *src, uint32_t bytes, uint32_t bar, int cold) {
    if (cold) {
        uint64_t policy;
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                     ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy) : "memory");
    } else {
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
    }
}

// Thread kPrefetchThread: copy tiles [t0, t0 + n) of a matrix of dtype with k inputs to dst, completing
// on the staging mbarrier. Quantised tiles go as one contiguous copy, f32/bf16 tiles one copy each at
// the padded stride. cold: with an L2 evict-first policy.
__device__ __noinline__ void stage_copy(const Smem &s, int dtype, const uint8_t *tiles, int k, int t0, int n, uint8_t *dst, int cold) {
    const size_t tb = tile_bytes(dtype, k), sst = staged_stride(dtype, k);
    const uint32_t bar = smem_addr(s.wbar);
    const uint8_t *src = tiles + (size_t)t0 * tb;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)(n * tb)) : "memory");
    if (sst == tb) bulk_copy(smem_addr(dst), src, (uint32_t)(n * tb), bar, cold);
    else
        for (int i = 0; i < n; i++) bulk_copy(smem_addr(dst + i * sst), src + i * tb, (uint32_t)tb, bar, cold);
}

// Every thread, after a __syncthreads that ends every read of dst: start the copy of tiles
// [t0, t0 + n) to dst, n = min(t1 - t0, cap) where cap is how many tiles fit (precomputed per matrix
// by the host); returns n. Only the issuing thread leaves the caller's code.
__device__ __forceinline__ int stage_issue(const Smem &s, int dtype, const uint8_t *tiles, int k, int t0, int t1, uint8_t *dst, int cap,
                                           int cold = 0) {
    const int n = t1 > t0 ? min(t1 - t0, cap) : 0;
    if (n > 0 && threadIdx.x == kPrefetchThread) stage_copy(s, dtype, tiles, k, t0, n, dst, cold);
    return n;
}

// The first failure of the launch: its code, and where it happened (the first CTA to record wins).
// With several GPUs the code is also stored into every other GPU's abort word, so their waits stop too.
__device__ __noinline__ void record_abort(const DecodeArgs &a, int code, int pos, int layer, int wait) {
    if (atomicCAS(a.hx.abort_flag, 0, code) == 0) {
        volatile int *w = a.hx.abort_flag;
        w[1] = blockIdx.x;
        w[2] = pos;
        w[3] = layer;
        w[4] = wait;
        for (int g = 0; g < a.sh.n_gpus; g++)
            if (g != a.sh.gpu) asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(a.sh.abort[g]), "r"(code) : "memory");
    }
}
__device__ __forceinline__ bool aborted(const DecodeArgs &a) { return *(volatile int *)a.hx.abort_flag != 0; }

// Poll phase parity par of the mbarrier at shared address bar until it completes (true), the time
// limit passes (false, the failure recorded as code/where) or, with abortable, another CTA has
// recorded a failure (false).
__device__ __forceinline__ bool mbar_wait_bounded(const DecodeArgs &a, uint32_t bar, uint32_t par, bool abortable, int code, int pos, int layer,
                                                  int wait) {
    uint64_t t0 = 0;
    for (int spins = 0;; spins++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(bar), "r"(par) : "memory");
        if (done) return true;
        if (spins == 0) {
            t0 = globaltimer_ns();
        } else if ((spins & 63) == 0) {
            if (abortable && aborted(a)) return false;
            if (globaltimer_ns() - t0 > a.hx.timeout_ns) {
                record_abort(a, code, pos, layer, wait);
                return false;
            }
        }
    }
}

// Every thread: wait for the outstanding copy (phase parity par of the mbarrier). Time-limited, and
// it stops early once a failure is recorded; the caller then goes on with whatever the buffer
// holds (the sampled position ends the launch). final: the wait before the CTA exits, which must
// see its own copy land (or its own limit pass) whatever other CTAs recorded.
__device__ __forceinline__ void stage_wait(const DecodeArgs &a, const Smem &s, uint32_t par, int pos, int layer, bool final = false) {
    mbar_wait_bounded(a, smem_addr(s.wbar), par, !final, kErrStageTimeout, pos, layer, kWaitStage);
}

// Exchange k (0-4) of the current layer has fully arrived in this CTA (phase parity par; every
// thread, time-limited, stopping early once a failure is recorded), then it is armed for the next
// layer: one arrival expecting `bytes`.
__device__ __noinline__ void xwait(const DecodeArgs &a, const Smem &s, int k, uint32_t par, uint32_t bytes, int pos, int layer) {
    const uint32_t bar = smem_addr(s.xbar + k);
    const bool done = mbar_wait_bounded(a, bar, par, true, kErrTimeout, pos, layer, kWaitQkv + k);
    __syncthreads();                                                      // every thread has seen this phase complete
    // Re-armed only when thread 0 saw the phase complete (an arrival on a phase that still has its
    // arrival is not allowed; after a failure the launch is ending anyway).
    if (threadIdx.x == 0 && done) asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// ---- Exchanges between GPUs (a model split over n_gpus > 1). Every layer step (position pos, layer
// l) has its own epoch; each element travels as one 8-byte word {value bits, epoch}, written with a
// single store, so a reader that sees the epoch it waits for has the value of that step, with no flag
// and no fence between them. Receive buffers alternate halves by step parity: a GPU writes step s + 2
// into a half only after every GPU has produced its part of step s + 1, which each produced after
// reading step s.
__device__ __forceinline__ uint32_t layer_step(const DecodeArgs &a, int pos, int l) { return (uint32_t)pos * (uint32_t)a.n_layers + (uint32_t)l; }
__device__ __forceinline__ int xlen(const DecodeArgs &a, int k) { return k == kXH ? a.ffn : a.dim; }
// The bytes of exchange k (-1: qkv) that this GPU's own CTAs deliver to each of its CTAs: 4 per value,
// or per 32-value block 40 (q8 bytes, scale, sum) for the q8 exchanges.
__device__ __forceinline__ uint32_t xbytes(const DecodeArgs &a, int k) {
    const uint32_t n = (uint32_t)(k < 0 ? a.sh.n_qkv_g : a.sh.len[k][a.sh.gpu]);
    if ((k == kXAttn && a.qx_attn == kXQ8) || (k == kXH && a.qx_h == kXQ8)) return n / kQB * 40u;
    return 4u * n;
}

// The q8 form of an exchange: src[0, n) (n a multiple of 32; this CTA's values g0.., g0 a multiple of
// 32), one warp per 32-value block: each lane takes one value, the block's maximum and sum come from
// warp shuffles (the prepare step's arithmetic, reference src/pack.c:101-122), the 32 bytes are packed
// by shuffles, and lane r (r < 16) stores the first 16 bytes and the scale into CTA r, lane 16 + r the
// last 16 bytes and the sum, with st.async completing on bar. src must be ready in shared memory.
__device__ __noinline__ void scatter_q8(const float *src, int g0, int n, const Prep &dst, unsigned long long *bar) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nblk = n / kQB, r = lane & 15, half = lane >> 4;
    uint32_t rb;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rb) : "r"((uint32_t)__cvta_generic_to_shared(bar)), "r"(r));
#pragma unroll 1
    for (int b = warp; b < nblk; b += (int)(blockDim.x >> 5)) {
        const float v = src[b * kQB + lane];
        const float av = fabsf(v);
        float m = av > 0.0f ? av : 0.0f;                                  // a NaN never raises the maximum
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float inv = m > 0.0f ? __fdiv_rn(127.0f, m) : 0.0f;
        const int q = (int8_t)__float2int_rn(__fmul_rn(v, inv));
        int sm = q;
#pragma unroll
        for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
        uint32_t w = (uint32_t)(q & 0xFF) << (8 * (lane & 3));              // byte lane & 3 of word lane >> 2
        w |= __shfl_xor_sync(0xffffffffu, w, 1);
        w |= __shfl_xor_sync(0xffffffffu, w, 2);
        uint32_t wv[4];
#pragma unroll
        for (int k = 0; k < 4; k++) wv[k] = __shfl_sync(0xffffffffu, w, 16 * half + 4 * k);
        const int bg = g0 / kQB + b;
        uint32_t ra, rs;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"((uint32_t)__cvta_generic_to_shared(dst.q8 + bg * kQB + 16 * half)), "r"(r));
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
                     ::"r"(ra), "r"(wv[0]), "r"(wv[1]), "r"(wv[2]), "r"(wv[3]), "r"(rb) : "memory");
        const uint32_t sw = half ? (uint32_t)sm : __float_as_uint(__fdiv_rn(m, 127.0f));
        const void *sd = half ? (const void *)(dst.sum + bg) : (const void *)(dst.scale + bg);
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rs) : "r"((uint32_t)__cvta_generic_to_shared(sd)), "r"(r));
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(rs), "r"(sw), "r"(rb) : "memory");
    }
}

// This CTA's part src[0, n) of exchanged vector k (elements [g0, g0 + n)) into every other GPU's
// receive buffer.
__device__ __noinline__ void peer_send(const DecodeArgs &a, int k, const float *src, int g0, int n, uint32_t step) {
    const int G = a.sh.n_gpus, me = a.sh.gpu;
    const uint64_t e = (uint64_t)(a.sh.epoch0 + step) << 32;
    const size_t half = (size_t)(step & 1u) * (size_t)xlen(a, k);
    #pragma unroll 1
    for (int j = threadIdx.x; j < n * (G - 1); j += blockDim.x) {
        const int p = j / n, i = j - p * n, g = p < me ? p : p + 1;
        unsigned long long *dst = a.sh.rx[g][k] + half + g0 + i;
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(e | __float_as_uint(src[i])) : "memory");
    }
}

// The other GPUs' slices of exchanged vector k into dst (shared memory), from this GPU's receive
// buffer: every thread polls its elements until their epoch is this step's (time-limited; stops
// early once a failure is recorded), then a barrier.
__device__ __noinline__ void peer_recv(const DecodeArgs &a, int k, float *dst, uint32_t step, int pos, int l) {
    const int G = a.sh.n_gpus, me = a.sh.gpu;
    const uint32_t e = a.sh.epoch0 + step;
    const unsigned long long *buf = a.sh.rx[me][k] + (size_t)(step & 1u) * (size_t)xlen(a, k);
    bool gave_up = false;
    uint64_t t0 = 0;
    int spins = 0;
    for (int g = 0; g < G && !gave_up; g++) {
        if (g == me) continue;
        const int lo = a.sh.lo[k][g], hi = lo + a.sh.len[k][g];
        #pragma unroll 1
        for (int i = lo + threadIdx.x; i < hi && !gave_up; i += blockDim.x) {
            for (;;) {
                uint64_t w;
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(buf + i) : "memory");
                if ((uint32_t)(w >> 32) == e) {
                    dst[i] = __uint_as_float((uint32_t)w);
                    break;
                }
                if (spins++ == 0) {
                    t0 = globaltimer_ns();
                } else if ((spins & 63) == 0) {
                    if (aborted(a)) { gave_up = true; break; }
                    if (globaltimer_ns() - t0 > a.hx.timeout_ns) {
                        record_abort(a, kErrTimeout, pos, l, kWaitPeerAttn + k);
                        gave_up = true;
                        break;
                    }
                }
            }
        }
    }
    __syncthreads();
}

// x = embedding row of tok, plus the learned position row when the file has one (reference
// src/engine.c:236-237, src/pack.c:55-62).
template <bool GPT2>
__device__ __noinline__ void embed_row(const DecodeArgs &a, int tok, int pos, float *x) {
    const uint8_t *row = a.embed + (size_t)tok * a.embed_row_bytes;
    #pragma unroll 1
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) {
        float v;
        if (a.dt_embed == DT_F32) v = __ldg((const float *)row + i);
        else if (a.dt_embed == DT_BF16) v = l3m_bf16_to_f32(ld_nc_u16(row + 2 * i));
        else {
            const int b = i >> 5, j = i & 31;
            if (a.dt_embed == DT_Q8) {
                const uint8_t *blk = row + b * 34;
                v = __fmul_rn(l3m_f16_to_f32(ld_nc_u16(blk)), (float)(int8_t)ld_nc_u8(blk + 2 + j));
            } else if (a.dt_embed == DT_Q4) {
                const uint8_t *blk = row + b * 18;
                uint8_t byte = ld_nc_u8(blk + 2 + (j & 15));
                int nib = j < 16 ? (byte & 15) : (byte >> 4);
                v = __fmul_rn(l3m_f16_to_f32(ld_nc_u16(blk)), (float)(nib - 8));
            } else {
                const uint8_t *blk = row + b * 17;
                uint8_t byte = ld_nc_u8(blk + 1 + (j & 15));
                int nib = j < 16 ? (byte & 15) : (byte >> 4);
                v = __fmul_rn(l3m_e8m0_half(ld_nc_u8(blk)), (float)l3m_mxfp4_value(nib));
            }
        }
        if (GPT2 && a.pos_embed) v = __fadd_rn(v, __ldg(a.pos_embed + (size_t)pos * a.dim + i));
        x[i] = v;
    }
    __syncthreads();
}

// Phase Q: this CTA's tiles of the q/k/v rows (biases added) -> s.y (the caller scatters into xq).
// ns tiles staged at the staging area's offset w_extra (phase parity par).
// The KV cache of (global) query head h: this GPU holds kv heads [kv_lo, kv_lo + n_kv_g).
__device__ __forceinline__ const uint16_t *kcache(const DecodeArgs &a, const LayerDev &L, int h) {
    return L.kc + (size_t)(h / a.hpk - a.sh.kv_lo) * a.ctx * a.hd;
}
__device__ __forceinline__ const uint16_t *vcache(const DecodeArgs &a, const LayerDev &L, int h) {
    return L.vc + (size_t)(h / a.hpk - a.sh.kv_lo) * a.hd * a.vstride;
}

// A head CTA's warps 1.. start the K/V copies of its attention (attend_prestage) while warp 0 runs
// the serial part of the rmsnorm (GPT2: the LayerNorm).
template <bool GPT2, bool TRACE>
__device__ __noinline__ void phase_qkv(const DecodeArgs &a, const LayerDev &L, const Role &role, const Smem &s, int ns, uint32_t par, int pos,
                                       int l, int tslot) {
    PreStage ps{};
    if (role.head0 >= 0) ps = PreStage{kcache(a, L, role.head0), vcache(a, L, role.head0), a.hd, a.vstride, pos, a.hd, s.kvbuf, s.vtbuf, a.attn_chunk};
    if (GPT2 && a.layernorm) layernorm_exact(s.x, s.wa, s.wab, a.dim, a.eps, s.xb, s.red, ps, L.dt_qkv, s.prep);
    else rmsnorm_exact(s.x, s.wa, a.dim, a.eps, s.xb, s.red, ps, L.dt_qkv, s.prep);   // and prepare
    trace<TRACE>(a, tslot, pos, l, 16);
    trace<TRACE>(a, tslot, pos, l, 17);
    if (ns) stage_wait(a, s, par, pos, l);
    trace<TRACE>(a, tslot, pos, l, 18);
    matvec_exact(L.dt_qkv, L.qkv, a.dim, role.qkv0, role.qkv1, s.prep, s.scratch, a.scratch_pairs, s.y, s.w + a.w_extra, ns);
    trace<TRACE>(a, tslot, pos, l, 19);
    // This GPU's qkv rows: q of its heads, then k and v of its kv heads (biases of the same rows).
    const int g0 = role.qkv0 * kTile, n = min(role.qkv1 * kTile, a.sh.n_qkv_g) - g0, nq = a.sh.n_heads_g * a.hd, nk = a.sh.n_kv_g * a.hd;
    if (L.bq) {
        const int q0 = a.sh.head_lo * a.hd, k0 = a.sh.kv_lo * a.hd;
        #pragma unroll 1
        for (int o = threadIdx.x; o < n; o += blockDim.x) {
            const int r = g0 + o;
            s.y[o] = __fadd_rn(s.y[o], __ldg(r < nq ? L.bq + q0 + r : r < nq + nk ? L.bk + k0 + (r - nq) : L.bv + k0 + (r - nq - nk)));
        }
        __syncthreads();
    }
}

// Phase A for query head h at position pos (xq complete): RoPE, this position's K/V row (stored by
// the first head of each kv group this GPU holds), attention -> every CTA's xa[h*hd, (h+1)*hd).
template <bool TRACE>
__device__ __noinline__ void phase_attention(const DecodeArgs &a, const LayerDev &L, const Smem &s, int h, int pos, bool prestaged, int l,
                                             int tslot) {
    const int tid = threadIdx.x, nth = blockDim.x, hd = a.hd, hl = h - a.sh.head_lo, kvl = h / a.hpk - a.sh.kv_lo;
    const int nq = a.sh.n_heads_g * hd, nk = a.sh.n_kv_g * hd;
    // q of this head (rotated) into y, k and v rows (rotated k) as bf16 into kcur / vcur and, by the
    // writer, into the cache: one pass, thread i taking input pair i (reference src/ops.c:29-40).
    float *y = s.y;
    const float *qs = s.xq + hl * hd, *ks = s.xq + nq + kvl * hd, *vs = s.xq + nq + nk + kvl * hd;
    uint16_t *kc = (uint16_t *)kcache(a, L, h), *vc = (uint16_t *)vcache(a, L, h);
    const bool writer = h % a.hpk == 0 || h == a.sh.head_lo;
#pragma unroll 1
    for (int i = tid; i < hd / 2; i += nth) {
        float q0 = qs[2 * i], q1 = qs[2 * i + 1], k0 = ks[2 * i], k1 = ks[2 * i + 1];
        if (a.rope) {
            const float2 c = s.rope[i];
            const float rq0 = __fmaf_rn(q0, c.x, -__fmul_rn(q1, c.y)), rq1 = __fmaf_rn(q0, c.y, __fmul_rn(q1, c.x));
            const float rk0 = __fmaf_rn(k0, c.x, -__fmul_rn(k1, c.y)), rk1 = __fmaf_rn(k0, c.y, __fmul_rn(k1, c.x));
            q0 = rq0; q1 = rq1; k0 = rk0; k1 = rk1;
        }
        y[2 * i] = q0;
        y[2 * i + 1] = q1;
        const uint16_t kb0 = l3m_f32_to_bf16(k0), kb1 = l3m_f32_to_bf16(k1);
        const uint16_t vb0 = l3m_f32_to_bf16(vs[2 * i]), vb1 = l3m_f32_to_bf16(vs[2 * i + 1]);
        s.kcur[2 * i] = kb0;
        s.kcur[2 * i + 1] = kb1;
        s.vcur[2 * i] = vb0;
        s.vcur[2 * i + 1] = vb1;
        if (writer) {
            *(uint32_t *)(kc + (size_t)pos * hd + 2 * i) = (uint32_t)kb0 | (uint32_t)kb1 << 16;
            vc[(size_t)(2 * i) * a.vstride + pos] = vb0;
            vc[(size_t)(2 * i + 1) * a.vstride + pos] = vb1;
        }
    }
    __syncthreads();
    trace<TRACE>(a, tslot, pos, l, 14);
    attend_exact<true>(y, kc, vc, hd, a.vstride, s.kcur, s.vcur, pos, hd, s.scores, s.att, s.red, a.etab, s.kvbuf, s.vtbuf,
                       a.attn_chunk, prestaged);
    trace<TRACE>(a, tslot, pos, l, 15);
    if (a.qx_attn == kXQ8) scatter_q8(s.att, h * hd, hd, s.pa, s.xbar + 1);
    else if (a.async_x && a.qx_attn == kXPrepBF16) scatter_tx<true>(s.att, s.xa, h * hd, hd, s.xbar + 1);
    else if (a.async_x) scatter_tx(s.att, s.xa, h * hd, hd, s.xbar + 1);
    else scatter(s.att, s.xa, h * hd, hd);
}

// Phase B: this CTA's tiles of wo over attn -> s.y (the caller scatters into xp; ns tiles staged at
// offset w_extra).
template <bool TRACE>
__device__ __noinline__ void phase_wo(const DecodeArgs &a, const LayerDev &L, const Role &role, const Smem &s, int ns, uint32_t par, int pos,
                                      int l, int tslot) {
    if (a.qx_attn == kXFloat) prepare(L.dt_wo, s.xa, a.dim, s.prep);     // else exchange 2 delivered it prepared
    trace<TRACE>(a, tslot, pos, l, 20);
    if (ns) stage_wait(a, s, par, pos, l);
    trace<TRACE>(a, tslot, pos, l, 21);
    matvec_exact(L.dt_wo, L.wo, a.dim, role.wo0, role.wo1, a.qx_attn != kXFloat ? s.pa : s.prep, s.scratch, a.scratch_pairs, s.y,
                 s.w + a.w_extra, ns);
    trace<TRACE>(a, tslot, pos, l, 22);
    const int g0 = (a.sh.d_off + role.wo0) * kTile, n = min((a.sh.d_off + role.wo1) * kTile, a.dim) - g0;
    if (L.bo) {
        #pragma unroll 1
        for (int o = threadIdx.x; o < n; o += blockDim.x) s.y[o] = __fadd_rn(s.y[o], __ldg(L.bo + g0 + o));
        __syncthreads();
    }
}

// Phase C: x += proj in every CTA; the ffn CTAs' tiles of up and gate -> s.y (up of the CTA's
// tiles, then gate; ns tiles of up, or of the interleaved up/gate, staged at offset 0).
template <bool GPT2, bool TRACE>
__device__ __noinline__ void phase_ffn(const DecodeArgs &a, const LayerDev &L, const Role &role, const Smem &s, int pos, int l, int tslot,
                                       int ns, uint32_t par) {
    #pragma unroll 1
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) s.x[i] = __fadd_rn(s.x[i], s.xp[i]);
    __syncthreads();
    if (role.ffn0 >= role.ffn1) return;
    if (GPT2 && a.layernorm) layernorm_exact(s.x, s.wf, s.wfb, a.dim, a.eps, s.xb, s.red, PreStage{}, L.dt_up, s.prep);
    else rmsnorm_exact(s.x, s.wf, a.dim, a.eps, s.xb, s.red, PreStage{}, L.dt_up, s.prep);   // and prepare
    trace<TRACE>(a, tslot, pos, l, 7);
    const int nf = role.ffn1 - role.ffn0;
    trace<TRACE>(a, tslot, pos, l, 26);
    if (ns) stage_wait(a, s, par, pos, l);
    trace<TRACE>(a, tslot, pos, l, 12);
    if (GPT2 && a.gelu) {                                                 // GPT-2: up only
        matvec_exact(L.dt_up, L.up, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, s.y, s.w, ns);
    } else if (!L.gate) {                                                 // up and gate packed per CTA: one pass
        matvec_exact(L.dt_up, L.up, a.dim, 2 * role.ffn0, 2 * role.ffn1, s.prep, s.scratch, a.scratch_pairs, s.y, s.w, ns);
    } else {
        matvec_exact(L.dt_up, L.up, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, s.y, s.w, ns);
        if (L.dt_gate != L.dt_up) prepare(L.dt_gate, s.xb, a.dim, s.prep);
        matvec_exact(L.dt_gate, L.gate, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, s.y + nf * kTile);
    }
    trace<TRACE>(a, tslot, pos, l, 13);
}

// The SiLU gate of phase C's up/gate results in s.y -> s.tmp (the caller scatters into xh); GPT2:
// GELU of up.
template <bool GPT2>
__device__ __noinline__ void ffn_gate(const DecodeArgs &a, const LayerDev &L, const Role &role, const Smem &s) {
    const int nf = role.ffn1 - role.ffn0, g0 = (a.sh.f_off + role.ffn0) * kTile, n = min((a.sh.f_off + role.ffn1) * kTile, a.ffn) - g0;
    #pragma unroll 1
    for (int o = threadIdx.x; o < n; o += blockDim.x) {
        const float up = L.b_up ? __fadd_rn(s.y[o], __ldg(L.b_up + g0 + o)) : s.y[o];
        s.tmp[o] = GPT2 && a.gelu ? gelu_tanh(up) : silu_mul(up, s.y[nf * kTile + o], a.etab);
    }
    __syncthreads();
}

// Phase D: this CTA's tiles of down over h -> s.y (the caller scatters into xd; ns tiles staged at
// offset 0).
template <bool TRACE>
__device__ __noinline__ void phase_down(const DecodeArgs &a, const LayerDev &L, const Role &role, const Smem &s, int ns, uint32_t par, int pos,
                                        int l, int tslot) {
    if (a.qx_h == kXFloat) prepare(L.dt_down, s.xh, a.ffn, s.prep);      // else exchange 4 delivered it prepared
    trace<TRACE>(a, tslot, pos, l, 23);
    if (ns) stage_wait(a, s, par, pos, l);
    trace<TRACE>(a, tslot, pos, l, 24);
    matvec_exact(L.dt_down, L.down, a.ffn, role.dn0, role.dn1, a.qx_h != kXFloat ? s.ph : s.prep, s.scratch, a.scratch_pairs, s.y, s.w, ns);
    trace<TRACE>(a, tslot, pos, l, 25);
    const int g0 = (a.sh.d_off + role.dn0) * kTile, n = min((a.sh.d_off + role.dn1) * kTile, a.dim) - g0;
    if (L.b_down) {
        #pragma unroll 1
        for (int o = threadIdx.x; o < n; o += blockDim.x) s.y[o] = __fadd_rn(s.y[o], __ldg(L.b_down + g0 + o));
        __syncthreads();
    }
}

// ---- Temperature sampling (reference engine.c:98-101, 283-287, 370-384, one rank): the weights
// p_i = expf((l_i - gmax) / T) (0 below -16), z = their sequential double sum, u = the next
// xorshift64* draw; the token is the first i whose running double sum exceeds u * z (the last
// index when none does: a NaN sum). Every nonzero weight is a float in [2^-24, 1], an integer
// number of 2^-47 units, so the running sums are computed exactly as 64-bit integers in parallel;
// the sequential double sum equals them until the first step whose exact sum is not a double
// (more than 53 significant bits: only after the sum passes 64 and only for weights below about
// 6e-5). Without such a step the draw is found in parallel from the exact sums; with one, one
// thread runs the reference's double chains over the stored weights (rare, slow, exact).
struct SampleIn {
    const float *logits;                 // [vocab], this position's
    float *probs;                        // [vocab] scratch: the weights
    int vocab;
    float temp, gmax;
    const uint32_t *etab;                // libm expf exception set
};

__device__ __forceinline__ double rand01(unsigned long long &st) {
    st ^= st >> 12;
    st ^= st << 25;
    st ^= st >> 27;
    return (double)((st * 0x2545F4914F6CDD1DULL) >> 11) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ unsigned long long weight_units(float p) {   // p * 2^47, exact
    return (unsigned long long)__fmul_rn(p, 140737488355328.0f);
}

__device__ __forceinline__ bool double_exact(unsigned long long e) {     // at most 53 significant bits
    const int bl = 64 - __clzll((long long)e);
    return bl <= 53 || (e & ((1ull << (bl - 53)) - 1)) == 0;
}

__device__ __forceinline__ void put_u64(float *d, unsigned long long v) {
    d[0] = __int_as_float((int)(uint32_t)v);
    d[1] = __int_as_float((int)(uint32_t)(v >> 32));
}
__device__ __forceinline__ unsigned long long get_u64(const float *d) {
    return (unsigned long long)(uint32_t)__float_as_int(d[0]) | (unsigned long long)(uint32_t)__float_as_int(d[1]) << 32;
}

// The smallest value of v over the CTA (every thread gets it); red: >= 8 ints of shared memory.
__device__ int cta_min(int v, int *red) {
    for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = min(m, red[w]);
    __syncthreads();
    return m;
}

// Every CTA of the cluster, in step; the same token returned in every CTA. xs: 3 x 16 x 4 floats of
// shared memory, written by every CTA of the cluster (distributed shared memory); tmp: 4 floats; red:
// 32 floats; stage: stage_n floats of shared memory for the one-thread fallback.
__device__ __noinline__ int sample_token(const SampleIn &in, float *xs, float *tmp, float *red, float *stage, int stage_n,
                                         unsigned long long &rng) {
    const int rank = (int)cg::this_cluster().block_rank(), tid = threadIdx.x, nth = blockDim.x, V = in.vocab;
    const double u = rand01(rng);
    const int lo = (int)((long long)rank * V / kClusterCtas), hi = (int)((long long)(rank + 1) * V / kClusterCtas);
    const int per = (hi - lo + nth - 1) / nth, i0 = min(hi, lo + tid * per), i1 = min(hi, i0 + per);
    // 1: the weights of this CTA's slice, their exact sum, NaN seen.
    unsigned long long tsum = 0;
    int nan = 0;
    for (int i = i0; i < i1; i++) {
        const float d = __fdiv_rn(__fsub_rn(ld_cg_f32(in.logits + i), in.gmax), in.temp);
        const float p = d < -16.0f ? 0.0f : l3m_expf_exact(d, in.etab);
        in.probs[i] = p;
        if (p != p) nan = 1;
        else tsum += weight_units(p);
    }
    unsigned long long incl = tsum;                                       // exclusive scan over threads (index order)
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
        if ((tid & 31) >= o) incl += n;
    }
    unsigned long long *wsum = (unsigned long long *)red;
    __syncthreads();
    if ((tid & 31) == 31) wsum[tid >> 5] = incl;
    const int anynan_cta = __syncthreads_or(nan);
    unsigned long long toff = incl - tsum, total = 0;
    for (int w = 0; w < nth >> 5; w++) {
        if (w < (tid >> 5)) toff += wsum[w];
        total += wsum[w];
    }
    if (tid == 0) { put_u64(tmp, total); tmp[2] = __int_as_float(anynan_cta); tmp[3] = 0.0f; }
    __syncthreads();
    scatter(tmp, xs, 4 * rank, 4);
    cluster_sync();
    unsigned long long base = 0, Z = 0;
    int anynan = 0;
    for (int c = 0; c < kClusterCtas; c++) {
        const unsigned long long t = get_u64(xs + 4 * c);
        if (c < rank) base += t;
        Z += t;
        anynan |= __float_as_int(xs[4 * c + 2]);
    }
    if (anynan) return V - 1;                                             // the same in every CTA
    // 2: the first step whose exact running sum is not a double.
    int first = 0x7FFFFFFF;
    {
        unsigned long long e = base + toff;
        for (int i = i0; i < i1; i++) {
            e += weight_units(in.probs[i]);
            if (!double_exact(e)) { first = i; break; }
        }
    }
    first = cta_min(first, (int *)red);
    if (tid == 0) { tmp[0] = __int_as_float(first); tmp[1] = tmp[2] = tmp[3] = 0.0f; }
    __syncthreads();
    scatter(tmp, xs + 4 * kClusterCtas, 4 * rank, 4);
    cluster_sync();
    int jr = 0x7FFFFFFF;
    for (int c = 0; c < kClusterCtas; c++) jr = min(jr, __float_as_int(xs[4 * kClusterCtas + 4 * c]));
    // 3: the draw.
    int tok = 0x7FFFFFFF;
    if (jr == 0x7FFFFFFF) {                                               // every running sum is a double: z = Z * 2^-47
        const double target = u * ((double)Z * 0x1p-47);
        unsigned long long e = base + toff;
        for (int i = i0; i < i1; i++) {
            e += weight_units(in.probs[i]);
            if ((double)e * 0x1p-47 > target) { tok = i; break; }
        }
        tok = cta_min(tok, (int *)red);
    } else if (rank == 0) {                                               // the reference's chains over the stored weights, by
        double z = 0.0, target = 0.0, c = 0.0;                            // thread 0, the CTA staging them in shared memory
        int *found = (int *)red;
        for (int pass = 0; pass < 2; pass++) {
            if (tid == 0) found[0] = 0x7FFFFFFF;
            for (int b0 = 0; b0 < V; b0 += stage_n) {
                const int n = min(stage_n, V - b0);
                __syncthreads();
                #pragma unroll 1
                for (int i = tid; i < n; i += nth) stage[i] = ld_cg_f32(in.probs + b0 + i);
                __syncthreads();
                if (tid == 0) {
                    if (pass == 0) {
                        for (int i = 0; i < n; i++) z += (double)stage[i];
                    } else if (found[0] == 0x7FFFFFFF) {
                        for (int i = 0; i < n; i++) {
                            c += (double)stage[i];
                            if (c > target) { found[0] = b0 + i; break; }
                        }
                    }
                }
            }
            if (pass == 0 && tid == 0) target = u * z;
        }
        __syncthreads();
        tok = found[0];
    }
    if (tid == 0) { tmp[0] = __int_as_float(tok); tmp[1] = tmp[2] = tmp[3] = 0.0f; }
    __syncthreads();
    scatter(tmp, xs + 8 * kClusterCtas, 4 * rank, 4);
    cluster_sync();
    int t = 0x7FFFFFFF;
    for (int c = 0; c < kClusterCtas; c++) t = min(t, __float_as_int(xs[8 * kClusterCtas + 4 * c]));
    return t == 0x7FFFFFFF ? V - 1 : t;
}

// The head matvec over this CTA's vocabulary tiles of the final x in s.x (logits kept for
// l3m_logits), this CTA's (max, index) in s.tmp[0..1] and, with several clusters, posted as its slot
// word for the tcount-th sampled position (a release store after the barrier that ends the logits
// stores). host_stop: the host's stop request (cluster 0, CTA 0 only). GPT2: the final LayerNorm.
// staged, ns: the first ns of the CTA's tiles are resident in shared memory (helper CTAs).
template <bool GPT2, bool TRACE>
__device__ __noinline__ void head_logits(const DecodeArgs &a, const Role &role, const Smem &s, int pos, int host_stop, int tslot,
                                         uint32_t tcount, const uint8_t *staged = nullptr, int ns = 0) {
    const int cta = blockIdx.x, tid = threadIdx.x, nth = blockDim.x;
    float best = -INFINITY;
    int best_i = -1;
    if (role.voc0 < role.voc1) {
        if (GPT2 && a.layernorm) layernorm_exact(s.x, s.wh, s.whb, a.dim, a.eps, s.xb, s.red, PreStage{}, a.dt_head, s.prep);
        else rmsnorm_exact(s.x, s.wh, a.dim, a.eps, s.xb, s.red, PreStage{}, a.dt_head, s.prep);   // and prepare
        trace<TRACE>(a, tslot, pos, a.n_layers, 3);
        trace<TRACE>(a, tslot, pos, a.n_layers, 4);
        matvec_exact(a.dt_head, a.head, a.dim, role.voc0, role.voc1, s.prep, s.scratch, a.scratch_pairs, s.y, staged, ns);
        trace<TRACE>(a, tslot, pos, a.n_layers, 5);
        float *lg = a.logits + (size_t)pos * a.vocab;
        const int g0 = (a.sh.v_off + role.voc0) * kTile, n = min((a.sh.v_off + role.voc1) * kTile, a.vocab) - g0;
        #pragma unroll 1
        for (int o = tid; o < n; o += nth) {
            const float v = s.y[o];
            lg[g0 + o] = v;
            if (v > best) { best = v; best_i = g0 + o; }                      // this thread's outputs rise with o
        }
        if (a.sh.n_gpus > 1) {                                            // GPU 0 keeps every logit (l3m_logits); with
            for (int t = 0; t < a.sh.n_gpus; t++) {                       // temperature sampling every GPU does
                if (t == a.sh.gpu || (t != 0 && !a.sh.all_logits)) continue;
                float *pl = a.sh.logits[t] + (size_t)pos * a.vocab + g0;
                #pragma unroll 1
                for (int o = tid; o < n; o += nth) pl[o] = s.y[o];
            }
            __threadfence_system();                                       // before the arrival that the vote follows
        }
    }
    // CTA argmax: the largest value, the lowest index among equals (reference engine.c:293-294).
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best || (ov == best && oi >= 0 && (best_i < 0 || oi < best_i))) { best = ov; best_i = oi; }
    }
    if ((tid & 31) == 0) { s.red[tid >> 5] = best; ((int *)s.red)[32 + (tid >> 5)] = best_i; }
    __syncthreads();
    if (tid == 0) {
        float m = -INFINITY;
        int mi = -1;
        for (int w = 0; w < nth / 32; w++) {
            const float v = s.red[w];
            const int vi = ((int *)s.red)[32 + w];
            if (v > m || (v == m && vi >= 0 && (mi < 0 || vi < mi))) { m = v; mi = vi; }
        }
        if (mi < 0) mi = (a.sh.v_off + role.voc0) * kTile;                   // an empty or all-NaN slice
        s.tmp[0] = m;                                                         // for a one-cluster launch
        s.tmp[1] = __int_as_float(mi);
        s.tmp[2] = __int_as_float(host_stop);
        if (a.grid > kClusterCtas && cta >= a.slot_lo) {
            const unsigned long long w = (unsigned long long)(head_epoch(tcount) << 24 | (uint32_t)mi) << 32 | __float_as_uint(m);
            asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(a.hx.slots + cta), "l"(w) : "memory");
        }
    }
    __syncthreads();
}

// Thread 0 of a helper: the next published position (epoch e of the x words): 1 and *pos, 0 when
// generation has ended (kHeadDone), -1 on the time limit or another CTA's abort. Sleeps between polls
// (the helpers wait through every layer of every position). The whole CTA learns the outcome.
__device__ __noinline__ int wait_published(const DecodeArgs &a, uint32_t e, int *pos) {
    __shared__ int res, where;
    if (threadIdx.x == 0) {
        const unsigned long long *p = a.hx.xw + a.dim;
        const uint64_t t0 = globaltimer_ns();
        int r = -1;
        for (int spins = 0;; spins++) {
            unsigned long long v;
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            if ((uint32_t)(v >> 32) == e) {
                r = (uint32_t)v == kHeadDone ? 0 : 1;
                where = (int)(uint32_t)v;
                break;
            }
            __nanosleep(32);
            if ((spins & 255) == 255) {
                if (globaltimer_ns() - t0 > a.hx.timeout_ns) { record_abort(a, kErrTimeout, -1, -1, kWaitHeadFlag); break; }
                if (aborted(a)) break;
            }
        }
        res = r;
    }
    __syncthreads();
    const int r = res;
    *pos = where;
    __syncthreads();
    return r;
}

// Every thread: x[i] = the value of x word i once it carries epoch e (the words are written without a
// fence, so each may land after the position word). Each thread issues the loads of up to 4 of its
// words at once (dim <= 1024 costs one round trip), then re-polls only words that are not there yet,
// with its own bounded wait. False on a failure.
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __noinline__ bool read_published_x(const DecodeArgs &a, uint32_t e, float *x, int pos) {
    const int nth = blockDim.x;
    bool ok = true;
#pragma unroll 1
    for (int i0 = threadIdx.x; i0 < a.dim && ok; i0 += 4 * nth) {
        unsigned long long v[4];
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u * nth < a.dim) v[u] = ld_relaxed_u64(a.hx.xw + i0 + u * nth);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int i = i0 + u * nth;
            if (i >= a.dim || !ok) continue;
            uint64_t t0 = 0;
            for (int spins = 0; (uint32_t)(v[u] >> 32) != e; spins++) {
                if (spins == 0) {
                    t0 = globaltimer_ns();
                } else if ((spins & 63) == 0) {
                    if (aborted(a)) { ok = false; break; }
                    if (globaltimer_ns() - t0 > a.hx.timeout_ns) { record_abort(a, kErrTimeout, pos, -1, kWaitHeadFlag); ok = false; break; }
                }
                v[u] = ld_relaxed_u64(a.hx.xw + i);
            }
            x[i] = __uint_as_float((uint32_t)v[u]);
        }
    }
    return __syncthreads_and(ok);
}

// Several GPUs: CTA 0 of each has its GPU's agreed (max, index, host stop, ok) in xt[0..3]. Its thread 0
// stores them into every GPU's vote buffer (two words, each with the sampled position's epoch, after
// a release that orders this GPU's logits stores before them), waits for every GPU's (acquire,
// time-limited), and reduces them in GPU order, the largest maximum and the first GPU among equals
// (the vocabulary order, reference src/engine.c:299-300); the host stop is GPU 0's, ok is all of
// them. The result goes to every CTA of cluster 0's xt[0..3] (the caller's cluster barrier follows).
__device__ __noinline__ void gpu_vote(const DecodeArgs &a, const Smem &s, uint32_t tcount, int pos) {
    if (threadIdx.x == 0) {
        const int G = a.sh.n_gpus, me = a.sh.gpu;
        const uint32_t e = a.sh.epoch0 + 0x40000000u + tcount;             // apart from the layer steps' epochs
        const size_t half = (size_t)(tcount & 1u) * kMaxShardGpus * 2;
        const uint32_t flags = (uint32_t)__float_as_int(s.xt[0]) & 0xFFFFFFu;
        const uint32_t word1 = flags | (__float_as_int(s.xt[1]) ? 1u << 24 : 0u) | (__float_as_int(s.xt[2]) ? 1u << 25 : 0u);
        const uint64_t w0 = (uint64_t)e << 32 | __float_as_uint(s.xt[3]), w1 = (uint64_t)e << 32 | word1;
        for (int g = 0; g < G; g++) {
            unsigned long long *v = a.sh.vote[g] + half + 2 * me;
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(v + 1), "l"(w1) : "memory");
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(v), "l"(w0) : "memory");
        }
        float gmax = -INFINITY;
        int next = 0, stop = 0, ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int g = 0; g < G; g++) {
            const unsigned long long *v = a.sh.vote[me] + half + 2 * g;
            uint64_t r0 = 0, r1 = 0;
            for (int spins = 0;; spins++) {
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(r0) : "l"(v) : "memory");
                if ((uint32_t)(r0 >> 32) == e) {
                    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(r1) : "l"(v + 1) : "memory");
                    if ((uint32_t)(r1 >> 32) == e) break;
                }
                if ((spins & 63) == 63 && (aborted(a) || globaltimer_ns() - t0 > a.hx.timeout_ns)) {
                    if (!aborted(a)) record_abort(a, kErrTimeout, pos, -1, kWaitPeerToken);
                    r0 = (uint64_t)e << 32 | __float_as_uint(-INFINITY);
                    r1 = 0;                                               // not ok
                    break;
                }
            }
            const float m = __uint_as_float((uint32_t)r0);
            const uint32_t f = (uint32_t)r1;
            if (m > gmax) { gmax = m; next = (int)(f & 0xFFFFFFu); }
            if (g == 0) stop = (f >> 24) & 1;
            ok &= (f >> 25) & 1;
        }
        s.tmp[0] = __int_as_float(next);
        s.tmp[1] = __int_as_float(stop);
        s.tmp[2] = __int_as_float(ok);
        s.tmp[3] = gmax;
    }
    __syncthreads();
    scatter(s.tmp, s.xt, 0, 4);
}

// A CTA outside cluster 0: between sampled positions it sleeps on the position word; for each published x it
// computes its vocabulary tiles. Its shared memory holds no layer state, so as many of its tiles as
// fit in the whole staging area are copied in once, at launch, and stay there for every position;
// the rest are pulled into L2 ahead of each use (cold: every tile, every position). Ends when
// cluster 0 writes kHeadDone (or on a failed wait).
template <bool GPT2, bool TRACE>
__device__ __noinline__ void head_helper(const DecodeArgs &a, const Role &role, const Smem &s, int cold, int tslot) {
    stage_init(s);
    const int nres = cold ? 0 : stage_issue(s, a.dt_head, a.head, a.dim, role.voc0, role.voc1, s.w, a.st_head);   // cold: read each time
    const size_t th = tile_bytes(a.dt_head, a.dim);
    const int rest0 = role.voc0 + nres;
    if (!cold && rest0 < role.voc1 && threadIdx.x == 0) prefetch_l2(a.head + rest0 * th, (size_t)(role.voc1 - rest0) * th);
    bool landed = nres == 0;
    for (uint32_t e = 1;; e++) {
        int pos;
        if (wait_published(a, e, &pos) <= 0) break;
        if (!read_published_x(a, e, s.x, pos)) break;
        cp_async_wait_all();                                              // the final norm's weights
        if (!landed) {                                                    // the resident tiles (first position only)
            stage_wait(a, s, 0, pos, -1);
            landed = true;
        }
        __syncthreads();
        trace<TRACE>(a, tslot, pos, a.n_layers, 0);
        head_logits<GPT2, TRACE>(a, role, s, pos, 0, tslot, e, s.w, nres);
        trace<TRACE>(a, tslot, pos, a.n_layers, 1);
        if (!cold && rest0 < role.voc1 && threadIdx.x == 0) prefetch_l2(a.head + rest0 * th, (size_t)(role.voc1 - rest0) * th);
    }
    if (!landed) stage_wait(a, s, 0, -1, -1, true);                       // no copy outlives the CTA
}

// Cold mode (reference src/engine.c:330-338): this CTA's share of the scratch buffer, cold_chunk bytes per
// copy into the attention-buffer part of the staging area (the bytes are never read), rounds of up to
// kFlushCopies copies on the staging mbarrier. The scratch, 1.5 x L2 over the cluster, displaces the
// weights from L2 before the next position starts.
constexpr int kFlushCopies = 8;
__device__ __noinline__ void cold_flush(const DecodeArgs &a, const Smem &s, int cta, uint32_t &wpar) {
    const unsigned long long share = a.cold_bytes / kClusterCtas, base = share * (unsigned long long)cta;
    const uint32_t chunk = (uint32_t)a.cold_chunk, bar = smem_addr(s.wbar);
    for (unsigned long long off = 0; off < share; off += (unsigned long long)kFlushCopies * chunk) {
        const int n = (int)min((unsigned long long)kFlushCopies, (share - off) / chunk);
        if (threadIdx.x == kPrefetchThread) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)n * chunk) : "memory");
            for (int i = 0; i < n; i++) bulk_copy(smem_addr(s.w), a.cold_buf + base + off + (unsigned long long)i * chunk, chunk, bar, 0);
        }
        stage_wait(a, s, wpar, -1, -1, true);
        wpar ^= 1;
        // Every thread has seen this round complete before the next one is armed; a recorded failure
        // ends the flush in every thread alike.
        if (__syncthreads_or(threadIdx.x == 0 && aborted(a))) break;
    }
}

// The weight-copy and exchange state carried from layer to layer: ns tiles of the outstanding copy,
// its mbarrier phase parity wpar, and the exchanges' phase parity xpar (one phase per layer).
struct LayerState {
    int ns;
    uint32_t wpar, xpar;
    unsigned long long wait_cyc;        // SM cycles spent in exchange and token waits (thread 0's count)
};

// One layer of position pos on cluster 0 (phases Q, A, B, C, D and the five exchanges), one
// out-of-line function so that the layer's code is one contiguous run.
template <bool GPT2, bool TRACE>
__device__ __noinline__ void run_layer(const DecodeArgs &a, const LayerDev *layers, int l, const Role &role, const Smem &s, int pos, bool last,
                                       int tslot, LayerState &st) {
    const int tid = threadIdx.x;
    const bool multi = a.sh.n_gpus > 1;
    int ns = st.ns;
    uint32_t wpar = st.wpar, xpar = st.xpar;
    const LayerDev &L = layers[l];
    cp_async_wait_all();                                          // this layer's norm weights and RoPE row
    __syncthreads();
    trace<TRACE>(a, tslot, pos, l, 0);
    if (l + 1 == a.n_layers) {
        if (last && role.voc0 < role.voc1 && tid == kPrefetchThread) {
            const size_t th = tile_bytes(a.dt_head, a.dim);
            prefetch_l2(a.head + role.voc0 * th, (size_t)(role.voc1 - role.voc0) * th);
        }
    }
    if (role.head0 >= 0 && role.qkv0 >= role.qkv1)               // K/V copies land during Q (else started by phase_qkv)
        attend_prestage<true>(kcache(a, L, role.head0), vcache(a, L, role.head0), a.hd, a.vstride, pos, a.hd, s.kvbuf, s.vtbuf,
                              a.attn_chunk);
    // Each phase: its matvec, its exchange, and the copy of the next phase's tiles (the staging area
    // is free once the matvec has read it). A copy landing in a CTA's shared memory delays the
    // exchange stores arriving there, so no copy is in flight while an exchange's stores are: the
    // wo and up/gate copies start once their exchange has arrived (each has the next phase's
    // prelude, 3 to 5 us, to land in); the next layer's qkv copy, which has only the norm (weights
    // from HBM when the model is larger than L2), starts right after the down exchange's stores;
    // the down copy is issued before the gate, which outlasts it.
    if (role.qkv0 < role.qkv1) phase_qkv<GPT2, TRACE>(a, L, role, s, ns, wpar, pos, l, tslot);   // Q
    if (ns) wpar ^= 1;
    trace<TRACE>(a, tslot, pos, l, 27);
    if (role.qkv0 < role.qkv1) {
        const int g0 = role.qkv0 * kTile, n = min(role.qkv1 * kTile, a.sh.n_qkv_g) - g0;
        if (a.async_x) scatter_tx(s.y, s.xq, g0, n, s.xbar);
        else scatter(s.y, s.xq, g0, n);
    }
    trace<TRACE>(a, tslot, pos, l, 1);
    long long w0 = clock64();
    if (a.async_x) xwait(a, s, 0, xpar, xbytes(a, -1), pos, l);   // 1: qkv (this GPU's heads)
    else cluster_sync();
    st.wait_cyc += clock64() - w0;
    ns = stage_issue(s, L.dt_wo, L.wo, a.dim, role.wo0, role.wo1, s.w + a.w_extra, L.st_wo, a.cold);
    trace<TRACE>(a, tslot, pos, l, 2);
    const uint32_t step = layer_step(a, pos, l);
    for (int h = role.head0; h >= 0 && h < a.sh.head_lo + a.sh.n_heads_g; h += kClusterCtas) {   // A
        phase_attention<TRACE>(a, L, s, h, pos, h == role.head0, l, tslot);
        if (multi) peer_send(a, kXAttn, s.att, h * a.hd, a.hd, step);
    }
    trace<TRACE>(a, tslot, pos, l, 3);
    w0 = clock64();
    if (a.async_x) xwait(a, s, 1, xpar, xbytes(a, kXAttn), pos, l);     // 2: attn
    else cluster_sync();
    if (multi) peer_recv(a, kXAttn, s.xa, step, pos, l);
    st.wait_cyc += clock64() - w0;
    trace<TRACE>(a, tslot, pos, l, 4);
    if (role.wo0 < role.wo1) phase_wo<TRACE>(a, L, role, s, ns, wpar, pos, l, tslot);   // B
    if (ns) wpar ^= 1;
    trace<TRACE>(a, tslot, pos, l, 28);
    if (role.wo0 < role.wo1) {
        const int g0 = (a.sh.d_off + role.wo0) * kTile, n = min((a.sh.d_off + role.wo1) * kTile, a.dim) - g0;
        if (a.async_x) scatter_tx(s.y, s.xp, g0, n, s.xbar + 2);
        else scatter(s.y, s.xp, g0, n);
        if (multi) peer_send(a, kXProj, s.y, g0, n, step);
    }
    trace<TRACE>(a, tslot, pos, l, 5);
    w0 = clock64();
    if (a.async_x) xwait(a, s, 2, xpar, xbytes(a, kXProj), pos, l);     // 3: proj
    else cluster_sync();
    if (multi) peer_recv(a, kXProj, s.xp, step, pos, l);
    st.wait_cyc += clock64() - w0;
    if (!L.gate && !(GPT2 && a.gelu)) ns = stage_issue(s, L.dt_up, L.up, a.dim, 2 * role.ffn0, 2 * role.ffn1, s.w, L.st_up, a.cold);
    else ns = stage_issue(s, L.dt_up, L.up, a.dim, role.ffn0, role.ffn1, s.w, L.st_up, a.cold);
    trace<TRACE>(a, tslot, pos, l, 6);
    phase_ffn<GPT2, TRACE>(a, L, role, s, pos, l, tslot, ns, wpar);      // C
    if (ns) wpar ^= 1;
    ns = stage_issue(s, L.dt_down, L.down, a.ffn, role.dn0, role.dn1, s.w, L.st_down, a.cold);
    trace<TRACE>(a, tslot, pos, l, 29);
    if (role.ffn0 < role.ffn1) {
        ffn_gate<GPT2>(a, L, role, s);
        const int g0 = (a.sh.f_off + role.ffn0) * kTile, n = min((a.sh.f_off + role.ffn1) * kTile, a.ffn) - g0;
        if (a.qx_h == kXQ8) scatter_q8(s.tmp, g0, n, s.ph, s.xbar + 3);
        else if (a.async_x && a.qx_h == kXPrepBF16) scatter_tx<true>(s.tmp, s.xh, g0, n, s.xbar + 3);
        else if (a.async_x) scatter_tx(s.tmp, s.xh, g0, n, s.xbar + 3);
        else scatter(s.tmp, s.xh, g0, n);
        if (multi) peer_send(a, kXH, s.tmp, g0, n, step);
    }
    // The next layer's norm weights (and the next position's RoPE row) while the rest runs.
    if (l + 1 < a.n_layers) stage_vectors<GPT2>(a, layers[l + 1], role, s, pos);
    else stage_vectors<GPT2>(a, layers[0], role, s, pos + 1);
    trace<TRACE>(a, tslot, pos, l, 8);
    w0 = clock64();
    if (a.async_x) xwait(a, s, 3, xpar, xbytes(a, kXH), pos, l);     // 4: h
    else cluster_sync();
    if (multi) peer_recv(a, kXH, s.xh, step, pos, l);
    st.wait_cyc += clock64() - w0;
    trace<TRACE>(a, tslot, pos, l, 9);
    if (role.dn0 < role.dn1) phase_down<TRACE>(a, L, role, s, ns, wpar, pos, l, tslot);   // D
    if (ns) wpar ^= 1;
    trace<TRACE>(a, tslot, pos, l, 30);
    if (role.dn0 < role.dn1) {
        const int g0 = (a.sh.d_off + role.dn0) * kTile, n = min((a.sh.d_off + role.dn1) * kTile, a.dim) - g0;
        if (a.async_x) scatter_tx(s.y, s.xd, g0, n, s.xbar + 4);
        else scatter(s.y, s.xd, g0, n);
        if (multi) peer_send(a, kXDown, s.y, g0, n, step);
    }
    if (l + 1 < a.n_layers || !a.cold) {                          // cold: the next position's first copy follows its flush
        const LayerDev &N = layers[l + 1 < a.n_layers ? l + 1 : 0];
        ns = stage_issue(s, N.dt_qkv, N.qkv, a.dim, role.qkv0, role.qkv1, s.w + a.w_extra, N.st_qkv, a.cold);
    } else {
        ns = 0;
    }
    trace<TRACE>(a, tslot, pos, l, 10);
    w0 = clock64();
    if (a.async_x) {                                              // 5: down
        xwait(a, s, 4, xpar, xbytes(a, kXDown), pos, l);
        xpar ^= 1u;
    } else {
        cluster_sync();
    }
    if (multi) peer_recv(a, kXDown, s.xd, step, pos, l);
    st.wait_cyc += clock64() - w0;
#pragma unroll 1
    for (int i = tid; i < a.dim; i += blockDim.x) s.x[i] = __fadd_rn(s.x[i], s.xd[i]);
    __syncthreads();
    trace<TRACE>(a, tslot, pos, l, 11);
    st.ns = ns;
    st.wpar = wpar;
    st.xpar = xpar;
}

// One instance per model family, so that neither costs the other registers or branches: GPT2
// (LayerNorm, learned positions, GELU: the GPT-2 family's layers); and per TRACE (the phase time
// stamps), so that the untraced instance carries none of their code. The layer loop's code has to
// stay inside the SM's instruction cache (between 96 and 128 KB on a B200: past that, every layer
// fetches its code again from L2), which is why thread-strided loops are not unrolled.
// The cluster shape is part of the kernel (__cluster_dims__), not only of the launch: a launch
// attribute alone is dropped by some launch paths (a profiler's replay ran this kernel as clusters of
// one CTA, which the entry check reports as kErrShape), while a compile-time shape holds for every
// launch of the function.
template <bool GPT2, bool TRACE>
__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kDecodeThreads, 1) decode_kernel(const DecodeArgs *__restrict__ ap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // The arguments, this CTA's role, every layer's pointers and the carved shared-memory pointers
    // live in shared memory for the whole launch.
    __shared__ DecodeArgs sh_args;
    __shared__ Role sh_role;
    __shared__ Smem sh_s;
    {
        // The launch shape this code assumes; anything else ends every CTA here, before any access
        // to another CTA's shared memory (which a cluster of another size would not have).
        uint32_t ncta, ncl;
        asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(ncta));
        asm("mov.u32 %0, %%nclusterid.x;" : "=r"(ncl));
        const int grid = ap->grid;
        if (ncta != (uint32_t)kClusterCtas || ncl * (uint32_t)kClusterCtas != gridDim.x || (int)gridDim.x != grid || gridDim.y != 1 ||
            gridDim.z != 1 || blockDim.x != (uint32_t)kDecodeThreads || blockDim.y != 1 || blockDim.z != 1) {
            if (blockIdx.x == 0 && threadIdx.x == 0) {
                Ctrl *c = ap->ctrl;
                c->where[0] = (int)ncta;
                c->where[1] = (int)ncl;
                c->where[2] = (int)gridDim.x;
                c->where[3] = (int)blockDim.x;
                c->error = kErrShape;
                __threadfence_system();
                c->done = 1;
            }
            return;
        }
    }
    if (threadIdx.x == 0) {
        sh_args = *ap;
        sh_role = ap->roles[blockIdx.x];
        if (ap->etab) prefetch_expf_table(ap->etab, blockIdx.x, gridDim.x);
    }
    __syncthreads();
    const DecodeArgs &a = sh_args;
    {
        const uint32_t *src = (const uint32_t *)ap->layers;
        uint32_t *dst = (uint32_t *)(smem_raw + a.sm_layers);
        #pragma unroll 1
        for (int i = threadIdx.x; i < a.n_layers * (int)(sizeof(LayerDev) / 4); i += blockDim.x) dst[i] = src[i];
    }
    const LayerDev *layers = (const LayerDev *)(smem_raw + a.sm_layers);
    if (threadIdx.x == 0) sh_s = carve(smem_raw, a);
    __syncthreads();
    const Smem &s = sh_s;
    const Role &role = sh_role;
    const int cta = blockIdx.x, tid = threadIdx.x;
    const long long cyc0 = clock64();                                     // CTA 0 keeps these for the statistics
    const unsigned long long gt0 = globaltimer_ns();
    const bool multi = a.sh.n_gpus > 1;
    const int tslot = a.trace_cta[0] == cta ? 0 : a.trace_cta[1] == cta ? 1 : -1;
    int n_gen = 0, tok = 0, pos = 0;
    uint32_t tcount = 0;
    unsigned long long rng = a.rng;                                       // advanced identically in every CTA of cluster 0
    bool ok = true;
    if (role.voc0 < role.voc1) {
        stage_f32(s.wh, a.norm, a.dim);
        if (GPT2 && a.layernorm) stage_f32(s.whb, a.norm_b, a.dim);
    }
    if (cta >= kClusterCtas) {                                            // the other clusters: head tiles only
        cp_async_commit();
        head_helper<GPT2, TRACE>(a, role, s, a.cold, tslot);
        cp_async_wait_all();
        return;
    }
    stage_vectors<GPT2>(a, layers[0], role, s, 0);
    stage_init(s);
    if (a.async_x && tid == 0) {
        const uint32_t bytes[5] = {xbytes(a, -1), xbytes(a, kXAttn), xbytes(a, kXProj), xbytes(a, kXH), xbytes(a, kXDown)};
        for (int k = 0; k < 5; k++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(s.xbar + k)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < 5; k++)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(s.xbar + k)), "r"(bytes[k]) : "memory");
    }
    // The staged-weight schedule: qkv and wo into [w_extra, w_bytes) (the attention buffers are live
    // from the layer top to the end of attention), up/gate and down from offset 0.
    LayerState st{0, 0, 0, 0};
    if (!a.cold) st.ns = stage_issue(s, layers[0].dt_qkv, layers[0].qkv, a.dim, role.qkv0, role.qkv1, s.w + a.w_extra, layers[0].st_qkv);
    unsigned long long cold_ns = 0;
    cluster_sync();                                                       // every CTA of the cluster has started

    for (pos = 0;; pos++) {
        const bool last = pos >= a.n_prompt - 1;
        if (pos < a.n_prompt) tok = a.prompt[pos];
        const bool stop_after = last && (n_gen >= a.max_new || pos + 1 >= a.ctx);   // reference engine.c:322, 352
        if (a.cold) {                                                     // evict the weights; not token time
            const unsigned long long f0 = globaltimer_ns();
            cold_flush(a, s, cta, st.wpar);
            cluster_sync();
            if (tid == 0) cold_ns += globaltimer_ns() - f0;
            st.ns = stage_issue(s, layers[0].dt_qkv, layers[0].qkv, a.dim, role.qkv0, role.qkv1, s.w + a.w_extra, layers[0].st_qkv, 1);
        }
        embed_row<GPT2>(a, tok, pos, s.x);
        for (int l = 0; l < a.n_layers; l++) run_layer<GPT2, TRACE>(a, layers, l, role, s, pos, last, tslot, st);
        if (!last) continue;                                              // the next position starts from its embedding
        ++tcount;
        // Publish x to every CTA of the launch (cluster 0's copies are identical) as epoch words, no
        // fence: each word carries its own epoch. Then this CTA's tiles, if it has any.
        if (cta == 0 && a.grid > kClusterCtas) {
            #pragma unroll 1
            for (int i = tid; i <= a.dim; i += blockDim.x) {
                const uint32_t v = i < a.dim ? __float_as_uint(s.x[i]) : (uint32_t)pos;
                asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a.hx.xw + i), "l"((unsigned long long)tcount << 32 | v) : "memory");
            }
        }
        trace<TRACE>(a, tslot, pos, a.n_layers, 0);
        int host_stop = 0;
        if (cta == 0 && tid == 0) host_stop = ld_relaxed_sys_i32((const int *)&a.ctrl->stop_request);
        if (a.grid == kClusterCtas || cta >= a.slot_lo) head_logits<GPT2, TRACE>(a, role, s, pos, host_stop, tslot, tcount);
        trace<TRACE>(a, tslot, pos, a.n_layers, 1);
        // One cluster: every CTA sends (max, index, host stop, no abort seen) to every CTA's xt[4 + 4 cta],
        // and after the barrier each reduces the same 16 slots in CTA order. Several clusters: CTA 0
        // waits for every posted slot word (one thread each, acquire: every slice of the logits is
        // written before its slot, also when nothing is sampled), reduces them in CTA order (the
        // vocabulary order, reference engine.c:299-300): the first CTA with the largest maximum; a slot
        // whose maximum is not above -inf (an empty or all-NaN slice) never wins, and with no winner
        // the token is 0 (the serial rule gmax = -inf; if (m > gmax) ...). The result goes to cluster
        // 0, so all 16 decide alike.
        if (a.grid == kClusterCtas) {
            if (tid == 0) s.tmp[3] = __int_as_float(*(volatile int *)a.hx.abort_flag == 0 ? 1 : 0);
            __syncthreads();
            scatter(s.tmp, s.xt, 4 + 4 * cta, 4);
        } else if (cta == 0) {
            const uint32_t e8 = head_epoch(tcount);
            float bm = -INFINITY;
            int bc = a.grid, bi = 0;
            bool good = true;
#pragma unroll 1
            for (int c = a.slot_lo + tid; c < a.grid && good; c += blockDim.x) {   // increasing c: strict > keeps the first
                unsigned long long w;
                uint64_t t0 = 0;
                for (int spins = 0;; spins++) {
                    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(a.hx.slots + c) : "memory");
                    if ((uint32_t)(w >> 56) == e8) break;
                    if (spins == 0) {
                        t0 = globaltimer_ns();
                    } else if ((spins & 63) == 0) {
                        if (aborted(a)) { good = false; break; }
                        if (globaltimer_ns() - t0 > a.hx.timeout_ns) { record_abort(a, kErrTimeout, pos, -1, kWaitHeadCount); good = false; break; }
                    }
                }
                const float m = __uint_as_float((uint32_t)w);
                if (good && m > bm) { bm = m; bc = c; bi = (int)((w >> 32) & 0xFFFFFFu); }
            }
            trace<TRACE>(a, tslot, pos, a.n_layers, 6);
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float om = __shfl_xor_sync(0xffffffffu, bm, o);
                const int oc = __shfl_xor_sync(0xffffffffu, bc, o), oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (om > bm || (om == bm && oc < bc)) { bm = om; bc = oc; bi = oi; }
            }
            const int nw = (int)(blockDim.x >> 5);                        // 8 warps: 24 of red's 64 words
            if ((tid & 31) == 0) { s.red[tid >> 5] = bm; ((int *)s.red)[nw + (tid >> 5)] = bc; ((int *)s.red)[2 * nw + (tid >> 5)] = bi; }
            const bool all_good = __syncthreads_and(good);
            if (tid == 0) {
                for (int w = 1; w < nw; w++) {
                    const float om = s.red[w];
                    const int oc = ((int *)s.red)[nw + w];
                    if (om > bm || (om == bm && oc < bc)) { bm = om; bc = oc; bi = ((int *)s.red)[2 * nw + w]; }
                }
                s.tmp[0] = __int_as_float(bc < a.grid ? bi : 0);
                s.tmp[1] = __int_as_float(host_stop);
                s.tmp[2] = __int_as_float(all_good && !*(volatile int *)a.hx.abort_flag ? 1 : 0);
                s.tmp[3] = bm;
            }
            __syncthreads();
            trace<TRACE>(a, tslot, pos, a.n_layers, 7);
            scatter(s.tmp, s.xt, 0, 4);
        }
        const long long w6 = clock64();
        cluster_sync();                                                   // 6: the sampled token
        if (a.grid == kClusterCtas) {
            float gmax = -INFINITY;
            int nx = 0, all = 1;
            for (int c = 0; c < kClusterCtas; c++) {
                const float *sl = s.xt + 4 + 4 * c;
                if (sl[0] > gmax) { gmax = sl[0]; nx = __float_as_int(sl[1]); }
                all &= __float_as_int(sl[3]);
            }
            __syncthreads();                                              // every thread has read the slots
            if (tid == 0) { s.xt[0] = __int_as_float(nx); s.xt[1] = s.xt[4 + 2]; s.xt[2] = __int_as_float(all); s.xt[3] = gmax; }
            __syncthreads();
        }
        if (multi) {                                                      // every GPU's (max, index): one agreed token
            cluster_sync();                                               // every CTA has its GPU's result in xt[0..3]
            if (cta == 0) gpu_vote(a, s, tcount, pos);
            cluster_sync();
        }
        st.wait_cyc += clock64() - w6;
        int next = __float_as_int(s.xt[0]);
        const int stop_req = __float_as_int(s.xt[1]);
        const float gmax_all = s.xt[3];
        if (!__float_as_int(s.xt[2])) { ok = false; break; }
        if (next < 0 || next >= a.vocab) {                                // never expected: the same in every CTA
            if (tid == 0) record_abort(a, kErrToken, pos, -1, next);
            ok = false;
            break;
        }
        trace<TRACE>(a, tslot, pos, a.n_layers, 2);
        if (stop_after) break;                                            // logits kept, nothing sampled (uniform)
        if (a.temp > 0.0f) {                                              // every CTA of cluster 0, in step
            const SampleIn in{a.logits + (size_t)pos * a.vocab, a.probs, a.vocab, a.temp, gmax_all, a.etab};
            next = sample_token(in, s.xt + 4 + 4 * kClusterCtas, s.tmp, s.red, (float *)s.scratch, 2 * a.scratch_pairs, rng);
        }
        tok = next;
        if (tok == a.eos || tok == a.bos) break;                          // reference engine.c:323-324
        n_gen++;
        if (cta == 0 && tid == 0 && a.sh.gpu == 0) {                      // GPU 0 streams the tokens
            a.tokens[n_gen - 1] = tok;
            __threadfence_system();
            a.ctrl->n_published = n_gen;
        }
        if (stop_req) break;
        // xt is rewritten at the next sampled position only after barriers 1-5, which every CTA
        // reaches after reading it here.
    }
    cp_async_wait_all();                                                  // no copy outlives the CTA
    if (st.ns) stage_wait(a, s, st.wpar, pos, -1, true);
    if (tid == 0) a.hx.stats[cta] = st.wait_cyc;
    cluster_sync();                                                       // no CTA leaves while others may write its memory
    if (cta == 0 && tid == 0) {
        if (a.grid > kClusterCtas)                                        // the helpers stop
            asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a.hx.xw + a.dim), "l"((unsigned long long)(tcount + 1) << 32 | kHeadDone) : "memory");
        unsigned long long wsum = 0;
        for (int c = 0; c < kClusterCtas; c++) wsum += ((volatile unsigned long long *)a.hx.stats)[c];
        a.ctrl->wait_cyc = wsum;
        a.ctrl->cold_ns = cold_ns;
        a.ctrl->cyc0 = (unsigned long long)cyc0;
        a.ctrl->gt0 = gt0;
        a.ctrl->cyc1 = (unsigned long long)clock64();
        a.ctrl->gt1 = globaltimer_ns();
        const int err = *(volatile int *)a.hx.abort_flag;
        a.ctrl->final_pos = pos;
        a.ctrl->n_gen = n_gen;
        for (int i = 0; i < 4; i++) a.ctrl->where[i] = ((volatile int *)a.hx.abort_flag)[1 + i];
        a.ctrl->error = ok ? 0 : (err ? err : kErrTimeout);
        __threadfence_system();
        a.ctrl->done = 1;
    }
}

// One draw of the sampler on its own (tests): a single 16-CTA cluster over logits already on the
// device; the maximum is found first (every CTA its slice, then an exchange).
__global__ void __launch_bounds__(kDecodeThreads, 1) sample_kernel(const float *logits, float *probs, int vocab, float temp,
                                                                  unsigned long long *rng_io, int *token, const uint32_t *etab) {
    __shared__ __align__(16) float xs[16 * kClusterCtas], xm[4 * kClusterCtas], tmp[4], red[64], stage[4096];
    const int rank = (int)cg::this_cluster().block_rank(), tid = threadIdx.x;
    const int lo = (int)((long long)rank * vocab / kClusterCtas), hi = (int)((long long)(rank + 1) * vocab / kClusterCtas);
    float m = -INFINITY;
    #pragma unroll 1
    for (int i = lo + tid; i < hi; i += blockDim.x) m = fmaxf(m, ld_cg_f32(logits + i));   // a NaN never wins
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float v = -INFINITY;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) v = fmaxf(v, red[w]);
        tmp[0] = v; tmp[1] = tmp[2] = tmp[3] = 0.0f;
    }
    __syncthreads();
    scatter(tmp, xm, 4 * rank, 4);
    cluster_sync();
    float gmax = -INFINITY;
    for (int c = 0; c < kClusterCtas; c++) gmax = fmaxf(gmax, xm[4 * c]);
    unsigned long long rng = *rng_io;
    const SampleIn in{logits, probs, vocab, temp, gmax, etab};
    const int t = sample_token(in, xs + 4, tmp, red, stage, 4096, rng);
    if (rank == 0 && tid == 0) { *token = t; *rng_io = rng; }
    cluster_sync();                                                       // no CTA leaves while others may write its memory
}

}  // namespace l3m

namespace {

// grid CTAs in clusters of kClusterCtas (the kernel's compile-time cluster shape), all resident at
// once (cooperative): the helper clusters wait on cluster 0 through global memory. at[1] carries the
// cluster shape for the occupancy query only (numAttrs 2); the launch itself uses numAttrs 1.
cudaLaunchConfig_t cluster_config(int grid, int smem_bytes, cudaLaunchAttribute *at) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(l3m::kDecodeThreads);
    cfg.dynamicSmemBytes = (size_t)smem_bytes;
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)l3m::kClusterCtas;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cfg;
}

using DecodeFn = void (*)(const l3m::DecodeArgs *);

// The kernel instance for a's model family, traced or not.
DecodeFn decode_instance(const l3m::DecodeArgs &a) {
    const bool gpt2 = a.layernorm || a.gelu || a.pos_embed != nullptr, traced = a.trace != nullptr;
    if (gpt2) return traced ? l3m::decode_kernel<true, true> : l3m::decode_kernel<true, false>;
    return traced ? l3m::decode_kernel<false, true> : l3m::decode_kernel<false, false>;
}

constexpr DecodeFn kDecodeInstances[4] = {l3m::decode_kernel<false, false>, l3m::decode_kernel<false, true>,
                                           l3m::decode_kernel<true, false>, l3m::decode_kernel<true, true>};

cudaError_t set_attributes(DecodeFn fn, int smem_bytes) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    return e;
}

}  // namespace

// a_dev: the arguments, already in device memory.
extern "C" int l3m_decode_launch(const l3m::DecodeArgs *a, const l3m::DecodeArgs *a_dev, void *stream) {
    if (!a_dev || !a->layers || !a->roles || !a->ctrl || !a->hx.abort_flag || !a->logits || !a->tokens) {   // never launch on an unset table
        fprintf(stderr, "l3m: decode launch: a device table is not set\n");
        return -1;
    }
    const DecodeFn fn = decode_instance(*a);
    cudaError_t e = set_attributes(fn, a->smem_bytes);
    if (e == cudaSuccess) {
        cudaLaunchAttribute at[2];
        cudaLaunchConfig_t cfg = cluster_config(a->grid, a->smem_bytes, at);
        cfg.stream = (cudaStream_t)stream;
        e = cudaLaunchKernelEx(&cfg, fn, a_dev);
    }
    if (e != cudaSuccess) {
        fprintf(stderr, "l3m: decode launch: %s\n", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

// The dynamic shared memory one decode CTA may use on the current device: the opt-in limit per block
// less the kernel's static shared memory.
extern "C" int l3m_decode_smem_budget(void) {
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return 0;
    int budget = optin;
    for (DecodeFn fn : kDecodeInstances) {                                // the least over the instances
        cudaFuncAttributes fa = {};
        if (cudaFuncGetAttributes(&fa, (const void *)fn) != cudaSuccess) return 0;
        budget = std::min(budget, optin - (int)fa.sharedSizeBytes);
    }
    return budget;
}

extern "C" int l3m_expf_table(const uint32_t **table);
extern "C" int l3m_error_msg(const char *msg);
extern "C" int l3m_error_cuda(int e, const char *what);

// One draw of the reference's sampler over device logits (include/l3m_kernels.h).
extern "C" L3M_API int l3m_sample_dev(const float *logits, int vocab, float temperature, uint64_t *rng_state, int32_t *token, float *scratch,
                                      void *stream) {
    if (vocab <= 0 || !(temperature > 0.0f)) return l3m_error_msg("l3m_sample_dev: vocab > 0 and temperature > 0");
    if (!logits || !rng_state || !token || !scratch) return l3m_error_msg("l3m_sample_dev: logits, rng_state, token and scratch are required");
    const uint32_t *etab;
    if (l3m_expf_table(&etab)) return -1;
    cudaError_t e = cudaFuncSetAttribute(l3m::sample_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute at[1];
        cfg.gridDim = dim3(l3m::kClusterCtas);
        cfg.blockDim = dim3(l3m::kDecodeThreads);
        cfg.stream = (cudaStream_t)stream;
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)l3m::kClusterCtas;
        at[0].val.clusterDim.y = at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, l3m::sample_kernel, logits, scratch, vocab, temperature, (unsigned long long *)rng_state, (int *)token,
                               etab);
    }
    return e == cudaSuccess ? 0 : l3m_error_cuda((int)e, "l3m_sample_dev");
}

// How many clusters of kClusterCtas CTAs with smem_bytes of shared memory each can be resident on
// the current device at once.
extern "C" int l3m_decode_occupancy(int smem_bytes) {
    int least = -1;
    for (DecodeFn fn : kDecodeInstances) {                                // the least over the instances
        if (set_attributes(fn, smem_bytes) != cudaSuccess) return 0;
        cudaLaunchAttribute at[2];
        cudaLaunchConfig_t cfg = cluster_config(l3m::kClusterCtas, smem_bytes, at);
        cfg.attrs = at + 1;                                               // the cluster shape, not cooperative
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, (const void *)fn, &cfg) != cudaSuccess) return 0;
        least = least < 0 ? n : std::min(least, n);
    }
    return least;
}
