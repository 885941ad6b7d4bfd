// The persistent decode kernel: one cooperative launch runs a whole l3m_generate call (prompt feed
// and greedy sampling) on one GPU, one CTA per SM. Replaces the reference's pinned thread pool and
// its four barriers per layer (src/engine.c:230-281, src/pool.c:111-123): no grid-wide barrier;
// a CTA waits only for the CTAs that produce what it reads.
//
// Per layer (step s, exchange buffers double-buffered by s % 2):
//   A  head CTAs: rmsnorm, q/k/v rows of their head, RoPE, KV row, attention  -> attn
//   B  wo CTAs:   wait attn, matvec                                           -> proj
//   C  all CTAs:  wait proj, x += proj, presence; ffn CTAs: rmsnorm, up and
//                 gate matvecs, SiLU gate                                      -> h
//   D  down CTAs: wait h, matvec                                              -> down
//   next layer / end of token: all CTAs wait down and every CTA's presence, x += down
// Presence makes every CTA finish reading step s before anyone writes step s + 2, so two buffers
// suffice. After the last prompt position each position ends with the head matvec, a per-CTA
// argmax and an all-to-all exchange of (max, index) that every CTA reduces in CTA order.
//
// An exchange is a float buffer plus an arrival counter. A producer writes its floats and adds its
// arrival (release); one thread of each consumer polls the counter (acquire, short sleeps) and
// then the whole CTA reads the floats once. A single polled word per exchange keeps L2 free for
// the CTAs doing the work. Presence is an arrival on the down counter.
#include <cstdio>
#include "ops.cuh"
#include "decode.cuh"

namespace l3m {

struct Smem {
    float *x, *xb, *tmp, *y, *att2, *scores, *att, *red, *wa, *wf, *wh;
    float2 *rope;
    uint16_t *kcur, *vcur, *kvbuf, *vtbuf;
    float2 *scratch;
    Prep prep;
};

__device__ __forceinline__ Smem carve(unsigned char *base, const DecodeArgs &a) {
    Smem s;
    s.x = (float *)(base + a.sm_x);
    s.xb = (float *)(base + a.sm_xb);
    s.tmp = (float *)(base + a.sm_tmp);
    s.y = (float *)(base + a.sm_y);
    s.att2 = (float *)(base + a.sm_y2);
    s.scores = (float *)(base + a.sm_scores);
    s.att = (float *)(base + a.sm_att);
    s.red = (float *)(base + a.sm_red);
    s.wa = (float *)(base + a.sm_wa);
    s.wf = (float *)(base + a.sm_wf);
    s.wh = (float *)(base + a.sm_wh);
    s.rope = (float2 *)(base + a.sm_rope);
    s.kcur = (uint16_t *)(base + a.sm_kv);
    s.vcur = s.kcur + a.hd;
    s.kvbuf = (uint16_t *)(base + a.sm_kvbuf);
    s.vtbuf = (uint16_t *)(base + a.sm_vt);
    s.scratch = (float2 *)(base + a.sm_scratch);
    s.prep.q8 = (int8_t *)(base + a.sm_q8);
    s.prep.scale = (float *)(base + a.sm_scale);
    s.prep.sum = (int32_t *)(base + a.sm_sum);
    s.prep.xf = (float *)(base + a.sm_xf);
    return s;
}

__device__ __forceinline__ void st_release_u32(uint32_t *p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_relaxed_f32(const float *p) {
    float v;
    asm volatile("ld.relaxed.gpu.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t *counter(const DecodeArgs &a, int x, uint32_t epoch) {
    return a.ctr + (x * 2 + (epoch & 1)) * 32;
}

// This CTA's part of exchange x at `epoch` is written (or, for presence, its reads are done):
// after the barrier one thread adds its arrival with release semantics, which covers every
// thread's writes before the barrier.
__device__ __forceinline__ void publish(const DecodeArgs &a, int x, uint32_t epoch) {
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter(a, x, epoch)) : "memory");
}

// Wait until exchange x has every arrival of `epoch` (counters only grow within a launch: the
// k-th use of a parity half expects k * arrivals). False on timeout or another CTA's abort.
__device__ __noinline__ bool wait_x(const DecodeArgs &a, int x, uint32_t epoch) {
    bool ok = true;
    if (threadIdx.x == 0) {
        const uint32_t *c = counter(a, x, epoch), want = ((epoch + 1) >> 1) * (uint32_t)a.arrivals[x];
        const uint64_t t0 = globaltimer_ns();
        for (int spins = 0;; spins++) {
            if (ld_acquire_u32(c) >= want) break;
            __nanosleep(32);
            if ((spins & 255) == 255) {
                if (globaltimer_ns() - t0 > a.timeout_ns) { atomicCAS(a.abort_flag, 0, kErrTimeout); ok = false; break; }
                if (*(volatile int *)a.abort_flag) { ok = false; break; }
            }
        }
    }
    return __syncthreads_and(ok);
}

// Read n exchanged floats into shared memory (after wait_x).
__device__ __forceinline__ void read_x(const float *src, int n, float *dst) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = ld_relaxed_f32(src + i);
    __syncthreads();
}

__device__ __forceinline__ float *xbuf(const DecodeArgs &a, int off, uint32_t epoch) {
    return a.xd + (epoch & 1) * a.xd_half + off;
}

__device__ __forceinline__ void trace(const DecodeArgs &a, int slot, int pos, int l, int ev) {
    if (a.trace && slot >= 0 && threadIdx.x == 0)
        a.trace[(((size_t)slot * a.ctx + pos) * (a.n_layers + 1) + l) * 16 + ev] = globaltimer_ns();
}

// Pull a CTA's weight tiles for layer l into L2 ahead of use (cp.async.bulk.prefetch: no registers,
// no completion to wait for). Every tile range is 16-byte aligned and a multiple of 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
    for (size_t o = 0; o < bytes; o += (1u << 20)) {
        const uint32_t n = (uint32_t)min(bytes - o, (size_t)1 << 20);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((const char *)p + o), "r"(n) : "memory");
    }
}

__device__ void prefetch_layer(const DecodeArgs &a, const LayerDev &L, const Role &r) {
    if (threadIdx.x != 0) return;
    const size_t tq = tile_bytes(L.dt_qkv, a.dim), to = tile_bytes(L.dt_wo, a.dim), tu = tile_bytes(L.dt_up, a.dim),
                 tg = tile_bytes(L.dt_gate, a.dim), td = tile_bytes(L.dt_down, a.ffn);
    if (r.head >= 0) prefetch_l2(L.qkv + (size_t)r.head * a.unit_tiles * tq, (size_t)a.unit_tiles * tq);
    if (r.wo0 < r.wo1) prefetch_l2(L.wo + r.wo0 * to, (size_t)(r.wo1 - r.wo0) * to);
    if (r.ffn0 < r.ffn1) {
        prefetch_l2(L.up + r.ffn0 * tu, (size_t)(r.ffn1 - r.ffn0) * tu);
        prefetch_l2(L.gate + r.ffn0 * tg, (size_t)(r.ffn1 - r.ffn0) * tg);
    }
    if (r.dn0 < r.dn1) prefetch_l2(L.down + r.dn0 * td, (size_t)(r.dn1 - r.dn0) * td);
}

// x = embedding row of tok (reference src/engine.c:236, src/pack.c:55-62).
__device__ __noinline__ void embed_row(const DecodeArgs &a, int tok, float *x) {
    const uint8_t *row = a.embed + (size_t)tok * a.embed_row_bytes;
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
        x[i] = v;
    }
    __syncthreads();
}

// Phase A for query head h of layer L at position pos: writes attn[h*hd, (h+1)*hd).
__device__ __noinline__ void phase_attention(const DecodeArgs &a, const LayerDev &L, const Role &role, int pos, float *attn, Smem &s,
                                             int tslot, int l) {
    const int tid = threadIdx.x, nth = blockDim.x, hd = a.hd, h = role.head, kvh = h / a.hpk;
    rmsnorm_exact(s.x, s.wa, a.dim, a.eps, s.xb, s.tmp, s.red);
    trace(a, tslot, pos, l, 8);
    prepare(L.dt_qkv, s.xb, a.dim, s.prep);
    trace(a, tslot, pos, l, 9);
    float *y = s.y;
    const uint8_t *unit = L.qkv + (size_t)h * a.unit_tiles * tile_bytes(L.dt_qkv, a.dim);
    matvec_exact(L.dt_qkv, unit, a.dim, 0, a.unit_tiles, s.prep, s.scratch, a.scratch_pairs, y);
    trace(a, tslot, pos, l, 10);
    if (L.bq) {
        for (int i = tid; i < hd; i += nth) {
            y[i] = __fadd_rn(y[i], __ldg(L.bq + h * hd + i));
            y[hd + i] = __fadd_rn(y[hd + i], __ldg(L.bk + kvh * hd + i));
            y[2 * hd + i] = __fadd_rn(y[2 * hd + i], __ldg(L.bv + kvh * hd + i));
        }
        __syncthreads();
    }
    if (a.rope) {
        rope_exact(y, hd, s.rope);
        rope_exact(y + hd, hd, s.rope);
    }
    uint16_t *kc = L.kc + (size_t)kvh * a.ctx * hd, *vc = L.vc + (size_t)kvh * hd * a.vstride;
    for (int i = tid; i < hd; i += nth) {
        const uint16_t kb = l3m_f32_to_bf16(y[hd + i]), vb = l3m_f32_to_bf16(y[2 * hd + i]);
        s.kcur[i] = kb;
        s.vcur[i] = vb;
        if (role.kv_writer) {
            kc[(size_t)pos * hd + i] = kb;
            vc[(size_t)i * a.vstride + pos] = vb;
        }
    }
    __syncthreads();
    trace(a, tslot, pos, l, 11);
    attend_exact<true>(y, kc, vc, hd, a.vstride, s.kcur, s.vcur, pos, hd, s.scores, s.att, s.red, a.elist, a.eindex, s.kvbuf, s.vtbuf,
                       a.attn_chunk);
    trace(a, tslot, pos, l, 12);
    for (int i = tid; i < hd; i += nth) attn[h * hd + i] = s.att[i];
}

__global__ void __launch_bounds__(kDecodeThreads, 1) decode_kernel(const DecodeArgs *__restrict__ ap) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // The arguments, this CTA's role and every layer's pointers live in shared memory for the whole
    // launch: reading them never waits on L1 misses behind the streamed weights.
    __shared__ DecodeArgs sh_args;
    __shared__ Role sh_role;
    if (threadIdx.x == 0) {
        sh_args = *ap;
        sh_role = ap->roles[blockIdx.x];
    }
    __syncthreads();
    const DecodeArgs &a = sh_args;
    {
        const uint32_t *src = (const uint32_t *)ap->layers;
        uint32_t *dst = (uint32_t *)(smem_raw + a.sm_layers);
        for (int i = threadIdx.x; i < a.n_layers * (int)(sizeof(LayerDev) / 4); i += blockDim.x) dst[i] = src[i];
    }
    const LayerDev *layers = (const LayerDev *)(smem_raw + a.sm_layers);
    __syncthreads();
    Smem s = carve(smem_raw, a);
    const int cta = blockIdx.x, tid = threadIdx.x, nth = blockDim.x;
    const Role &role = sh_role;
    int tslot = -1;
    for (int i = 0; i < 4; i++) if (a.trace_cta[i] == cta) tslot = i;
    uint32_t step = 0, tcount = 0;
    int n_gen = 0, tok = 0, pos = 0, err = 0;
    bool ok = true;

    for (pos = 0;; pos++) {
        const bool last = pos >= a.n_prompt - 1;
        if (pos < a.n_prompt) tok = a.prompt[pos];
        const bool stop_after = last && (n_gen >= a.max_new || pos + 1 >= a.ctx);   // reference engine.c:322, 352
        embed_row(a, tok, s.x);
        for (int l = 0; l < a.n_layers && ok; l++) {
            ++step;
            const LayerDev &L = layers[l];
            if (l + 1 < a.n_layers) prefetch_layer(a, layers[l + 1], role);
            else {
                prefetch_layer(a, layers[0], role);
                if (last && role.voc0 < role.voc1 && threadIdx.x == 0) {
                    const size_t th = tile_bytes(a.dt_head, a.dim);
                    prefetch_l2(a.head + role.voc0 * th, (size_t)(role.voc1 - role.voc0) * th);
                }
            }
            // This layer's small vectors into shared memory while the exchange below is awaited.
            if (role.head >= 0) {
                stage_f32(s.wa, L.attn_norm, a.dim);
                if (a.rope) stage_f32((float *)s.rope, (const float *)(a.rope + (size_t)pos * (a.hd / 2)), a.hd);
            }
            if (role.ffn0 < role.ffn1) stage_f32(s.wf, L.ffn_norm, a.dim);
            if (l + 1 == a.n_layers && last && role.voc0 < role.voc1) stage_f32(s.wh, a.norm, a.dim);
            cp_async_commit();
            if (l > 0) {
                if (!(ok = wait_x(a, kXDown, step - 1))) break;
                read_x(xbuf(a, a.d_down, step - 1), a.dim, s.tmp);
                for (int i = tid; i < a.dim; i += nth) s.x[i] = __fadd_rn(s.x[i], s.tmp[i]);
            }
            cp_async_wait_all();
            __syncthreads();
            trace(a, tslot, pos, l, 0);
            if (role.head >= 0) {                                            // A
                phase_attention(a, L, role, pos, xbuf(a, a.d_attn, step), s, tslot, l);
                publish(a, kXAttn, step);
            }
            trace(a, tslot, pos, l, 1);
            if (role.wo0 < role.wo1) {                                       // B
                if (!(ok = wait_x(a, kXAttn, step))) break;
                trace(a, tslot, pos, l, 2);
                read_x(xbuf(a, a.d_attn, step), a.dim, s.xb);
                prepare(L.dt_wo, s.xb, a.dim, s.prep);
                matvec_exact(L.dt_wo, L.wo, a.dim, role.wo0, role.wo1, s.prep, s.scratch, a.scratch_pairs, s.y);
                float *out = xbuf(a, a.d_proj, step);
                const int g0 = role.wo0 * kTile, n = min(role.wo1 * kTile, a.dim) - g0;
                for (int o = tid; o < n; o += nth) out[g0 + o] = L.bo ? __fadd_rn(s.y[o], __ldg(L.bo + g0 + o)) : s.y[o];
                publish(a, kXProj, step);
            }
            if (!(ok = wait_x(a, kXProj, step))) break;                      // C
            trace(a, tslot, pos, l, 3);
            read_x(xbuf(a, a.d_proj, step), a.dim, s.tmp);
            for (int i = tid; i < a.dim; i += nth) s.x[i] = __fadd_rn(s.x[i], s.tmp[i]);
            publish(a, kXDown, step);                                       // presence: done reading step - 1
            if (role.ffn0 < role.ffn1) {
                rmsnorm_exact(s.x, s.wf, a.dim, a.eps, s.xb, s.tmp, s.red);
                trace(a, tslot, pos, l, 13);
                prepare(L.dt_up, s.xb, a.dim, s.prep);
                matvec_exact(L.dt_up, L.up, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, s.y);
                trace(a, tslot, pos, l, 14);
                if (L.dt_gate != L.dt_up) prepare(L.dt_gate, s.xb, a.dim, s.prep);
                matvec_exact(L.dt_gate, L.gate, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, s.att2);
                trace(a, tslot, pos, l, 15);
                float *out = xbuf(a, a.d_h, step);
                const int g0 = role.ffn0 * kTile, n = min(role.ffn1 * kTile, a.ffn) - g0;
                for (int o = tid; o < n; o += nth) {
                    const float up = L.b_up ? __fadd_rn(s.y[o], __ldg(L.b_up + g0 + o)) : s.y[o];
                    out[g0 + o] = silu_mul(up, s.att2[o], a.elist, a.eindex);
                }
                publish(a, kXH, step);
            }
            trace(a, tslot, pos, l, 4);
            if (role.dn0 < role.dn1) {                                       // D
                if (!(ok = wait_x(a, kXH, step))) break;
                trace(a, tslot, pos, l, 5);
                read_x(xbuf(a, a.d_h, step), a.ffn, s.xb);
                prepare(L.dt_down, s.xb, a.ffn, s.prep);
                matvec_exact(L.dt_down, L.down, a.ffn, role.dn0, role.dn1, s.prep, s.scratch, a.scratch_pairs, s.y);
                float *out = xbuf(a, a.d_down, step);
                const int g0 = role.dn0 * kTile, n = min(role.dn1 * kTile, a.dim) - g0;
                for (int o = tid; o < n; o += nth) out[g0 + o] = L.b_down ? __fadd_rn(s.y[o], __ldg(L.b_down + g0 + o)) : s.y[o];
                publish(a, kXDown, step);
            }
            trace(a, tslot, pos, l, 6);
        }
        if (!ok) break;
        if (!(ok = wait_x(a, kXDown, step))) break;
        read_x(xbuf(a, a.d_down, step), a.dim, s.tmp);
        for (int i = tid; i < a.dim; i += nth) s.x[i] = __fadd_rn(s.x[i], s.tmp[i]);
        __syncthreads();
        trace(a, tslot, pos, a.n_layers, 0);
        if (!last) continue;

        // Head: logits for this position and this CTA's share of the argmax.
        ++tcount;
        int host_stop = 0;
        if (cta == 0 && tid == 0) host_stop = ld_relaxed_sys_i32((const int *)&a.ctrl->stop_request);
        float best = -INFINITY;
        int best_i = -1;
        if (role.voc0 < role.voc1) {
            rmsnorm_exact(s.x, s.wh, a.dim, a.eps, s.xb, s.tmp, s.red);
            prepare(a.dt_head, s.xb, a.dim, s.prep);
            matvec_exact(a.dt_head, a.head, a.dim, role.voc0, role.voc1, s.prep, s.scratch, a.scratch_pairs, s.y);
            float *lg = a.logits + (size_t)pos * a.vocab;
            const int g0 = role.voc0 * kTile, n = min(role.voc1 * kTile, a.vocab) - g0;
            for (int o = tid; o < n; o += nth) {
                const float v = s.y[o];
                lg[g0 + o] = v;
                if (v > best) { best = v; best_i = g0 + o; }                  // this thread's outputs rise with o
            }
        }
        trace(a, tslot, pos, a.n_layers, 1);
        if (stop_after) break;                                              // logits kept, nothing sampled
        // CTA argmax: the largest value, the lowest index among equals (reference engine.c:293-294).
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best || (ov == best && oi >= 0 && (best_i < 0 || oi < best_i))) { best = ov; best_i = oi; }
        }
        if ((tid & 31) == 0) { s.red[tid >> 5] = best; ((int *)s.red)[32 + (tid >> 5)] = best_i; }
        __syncthreads();
        float *tx = xbuf(a, a.d_tok, tcount);
        if (tid == 0) {
            float m = -INFINITY;
            int mi = -1;
            for (int w = 0; w < nth / 32; w++) {
                const float v = s.red[w];
                const int vi = ((int *)s.red)[32 + w];
                if (v > m || (v == m && vi >= 0 && (mi < 0 || vi < mi))) { m = v; mi = vi; }
            }
            if (mi < 0) mi = role.voc0 * kTile;                               // an empty or all-NaN slice
            tx[3 * cta] = m;
            tx[3 * cta + 1] = __int_as_float(mi);
            tx[3 * cta + 2] = __int_as_float(host_stop);
        }
        publish(a, kXTok, tcount);
        if (!(ok = wait_x(a, kXTok, tcount))) break;
        read_x(tx, 3 * a.grid, s.scores);
        // Global argmax over the CTAs in vocabulary order (reference engine.c:299-300), same in every CTA.
        float gmax = -INFINITY;
        int next = 0;
        for (int c = 0; c < a.grid; c++) {
            if (s.scores[3 * c] > gmax) { gmax = s.scores[3 * c]; next = __float_as_int(s.scores[3 * c + 1]); }
        }
        const int stop_req = __float_as_int(s.scores[2]);
        __syncthreads();
        trace(a, tslot, pos, a.n_layers, 2);
        tok = next;
        if (tok == a.eos || tok == a.bos) break;                              // reference engine.c:323-324
        n_gen++;
        if (cta == 0 && tid == 0) {
            a.tokens[n_gen - 1] = tok;
            __threadfence_system();
            a.ctrl->n_published = n_gen;
        }
        if (stop_req) break;
    }
    cp_async_wait_all();                                                    // no copy outlives the CTA
    if (!ok) err = *(volatile int *)a.abort_flag;
    if (cta == 0 && tid == 0) {
        a.ctrl->final_pos = pos;
        a.ctrl->n_gen = n_gen;
        a.ctrl->error = err ? err : (ok ? 0 : kErrTimeout);
        __threadfence_system();
        a.ctrl->done = 1;
    }
}

}  // namespace l3m

// a_dev: the arguments, already in device memory.
extern "C" int l3m_decode_launch(const l3m::DecodeArgs *a, const l3m::DecodeArgs *a_dev, void *stream) {
    void *args[] = {(void *)&a_dev};
    cudaError_t e = cudaFuncSetAttribute(l3m::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, a->smem_bytes);
    if (e == cudaSuccess)
        e = cudaLaunchCooperativeKernel((const void *)l3m::decode_kernel, dim3(a->grid), dim3(l3m::kDecodeThreads), args,
                                        (size_t)a->smem_bytes, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        fprintf(stderr, "l3m: decode launch: %s\n", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int l3m_decode_occupancy(int smem_bytes) {
    int n = 0;
    if (cudaFuncSetAttribute(l3m::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, l3m::decode_kernel, l3m::kDecodeThreads, smem_bytes) != cudaSuccess) return 0;
    return n;
}
