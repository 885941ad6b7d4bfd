// The persistent decode kernel: one cooperative launch runs a whole l3m_generate call (prompt feed
// and greedy sampling) on one GPU, one CTA per SM. Replaces the reference's pinned thread pool and
// its four barriers per layer (src/engine.c:230-281, src/pool.c:111-123): each phase's outputs go
// out as flagged 64-bit slots, and a CTA waits only for the slots it reads. A phase therefore
// costs one round trip through L2 instead of a barrier plus a copy.
//
// Per layer (step s, slots double-buffered by s % 2):
//   A  head CTAs: rmsnorm, q/k/v rows of their head, RoPE, KV row, attention  -> attn slots
//   B  wo CTAs:   wait attn, matvec                                           -> proj slots
//   C  all CTAs:  wait proj, x += proj, post presence; ffn CTAs: rmsnorm,
//                 up and gate matvecs, SiLU gate                               -> h slots
//   D  down CTAs: wait h, matvec                                              -> down slots
//   next layer / end of token: all CTAs wait down + every CTA's presence, x += down
// The presence slots make every CTA finish reading step s before anyone writes step s + 2, so two
// buffers suffice. After the last prompt position each position ends with the head matvec, a
// per-CTA argmax and an all-to-all exchange of (max, index) that every CTA reduces in CTA order.
#include <cstdio>
#include "ops.cuh"
#include "decode.cuh"

namespace l3m {

struct Smem {
    float *x, *xb, *tmp, *y, *scores, *att, *red;
    uint16_t *kcur, *vcur;
    float2 *scratch;
    Prep prep;
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
    s.kcur = (uint16_t *)(base + a.sm_kv);
    s.vcur = s.kcur + a.hd;
    s.scratch = (float2 *)(base + a.sm_scratch);
    s.prep.q8 = (int8_t *)(base + a.sm_q8);
    s.prep.scale = (float *)(base + a.sm_scale);
    s.prep.sum = (int32_t *)(base + a.sm_sum);
    s.prep.xf = (float *)(base + a.sm_xf);
    return s;
}

// Wait until slots[0, n) carry `epoch`; values go to dst (may be NULL). Every thread polls its
// own slots, all outstanding loads in flight together. False on timeout or another CTA's abort.
__device__ bool wait_slots(const uint64_t *slots, int n, uint32_t epoch, float *dst, const DecodeArgs &a) {
    constexpr int kMax = 8;
    const int tid = threadIdx.x, nth = blockDim.x;
    bool ok = true;
    for (int base = 0; base < n; base += kMax * nth) {
        uint32_t pending = 0;
#pragma unroll
        for (int j = 0; j < kMax; j++) if (base + tid + j * nth < n) pending |= 1u << j;
        const uint64_t t0 = globaltimer_ns();
        int spins = 0;
        while (pending) {
#pragma unroll
            for (int j = 0; j < kMax; j++) {
                if (!(pending >> j & 1)) continue;
                const int i = base + tid + j * nth;
                const uint64_t w = slot_get(slots + i);
                if (slot_epoch(w) == epoch) {
                    if (dst) dst[i] = slot_value(w);
                    pending &= ~(1u << j);
                }
            }
            if (pending && (++spins & 255) == 0) {
                if (globaltimer_ns() - t0 > a.timeout_ns) { atomicCAS(a.abort_flag, 0, kErrTimeout); ok = false; break; }
                if (*(volatile int *)a.abort_flag) { ok = false; break; }
            }
        }
        if (!ok) break;
    }
    return __syncthreads_and(ok);
}

__device__ __forceinline__ void put(uint64_t *slot, float v, uint32_t epoch) { slot_put(slot, slot_word(v, epoch)); }

// x = embedding row of tok (reference src/engine.c:236, src/pack.c:55-62).
__device__ void embed_row(const DecodeArgs &a, int tok, float *x) {
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

// Phase A for query head h of layer L at position pos.
__device__ void phase_attention(const DecodeArgs &a, const LayerDev &L, const Role &role, int pos, uint64_t *ex_attn,
                                uint32_t step, Smem &s) {
    const int tid = threadIdx.x, nth = blockDim.x, hd = a.hd, h = role.head, kvh = h / a.hpk;
    rmsnorm_exact(s.x, L.attn_norm, a.dim, a.eps, s.xb, s.tmp, s.red);
    prepare(L.dt_qkv, s.xb, a.dim, s.prep);
    float *y = s.y;
    const uint8_t *unit = L.qkv + (size_t)h * a.unit_tiles * tile_bytes(L.dt_qkv, a.dim);
    matvec_exact(L.dt_qkv, unit, a.dim, 0, a.unit_tiles, s.prep, s.scratch, a.scratch_pairs, [&](int o, float v) { y[o] = v; });
    if (L.bq) {
        for (int i = tid; i < hd; i += nth) {
            y[i] = __fadd_rn(y[i], __ldg(L.bq + h * hd + i));
            y[hd + i] = __fadd_rn(y[hd + i], __ldg(L.bk + kvh * hd + i));
            y[2 * hd + i] = __fadd_rn(y[2 * hd + i], __ldg(L.bv + kvh * hd + i));
        }
        __syncthreads();
    }
    if (a.rope) {
        rope_exact(y, hd, a.rope + (size_t)pos * (hd / 2));
        rope_exact(y + hd, hd, a.rope + (size_t)pos * (hd / 2));
    }
    uint16_t *kc = L.kc + (size_t)kvh * a.ctx * hd, *vc = L.vc + (size_t)kvh * a.ctx * hd;
    for (int i = tid; i < hd; i += nth) {
        const uint16_t kb = l3m_f32_to_bf16(y[hd + i]), vb = l3m_f32_to_bf16(y[2 * hd + i]);
        s.kcur[i] = kb;
        s.vcur[i] = vb;
        if (role.kv_writer) {
            kc[(size_t)pos * hd + i] = kb;
            vc[(size_t)pos * hd + i] = vb;
        }
    }
    __syncthreads();
    attend_exact(y, kc, vc, hd, s.kcur, s.vcur, pos, hd, s.scores, s.att, s.red, a.elist, a.eindex);
    for (int i = tid; i < hd; i += nth) put(ex_attn + h * hd + i, s.att[i], step);
}

__global__ void __launch_bounds__(512, 1) decode_kernel(const DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem s = carve(smem_raw, a);
    const int cta = blockIdx.x, tid = threadIdx.x, nth = blockDim.x;
    const Role role = a.roles[cta];
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
            const LayerDev L = a.layers[l];
            uint64_t *ex = a.ex + (step & 1) * a.ex_half, *ex_prev = a.ex + ((step - 1) & 1) * a.ex_half;
            if (l > 0) {
                ok = wait_slots(ex_prev + a.off_down, a.dim, step - 1, s.tmp, a) && wait_slots(ex_prev + a.off_pres, a.grid, step - 1, nullptr, a);
                if (!ok) break;
                for (int i = tid; i < a.dim; i += nth) s.x[i] = __fadd_rn(s.x[i], s.tmp[i]);
                __syncthreads();
            }
            if (role.head >= 0) phase_attention(a, L, role, pos, ex + a.off_attn, step, s);
            if (role.wo0 < role.wo1) {                                       // B
                if (!(ok = wait_slots(ex + a.off_attn, a.dim, step, s.xb, a))) break;
                prepare(L.dt_wo, s.xb, a.dim, s.prep);
                uint64_t *out = ex + a.off_proj;
                const int g0 = role.wo0 * kTile;
                matvec_exact(L.dt_wo, L.wo, a.dim, role.wo0, role.wo1, s.prep, s.scratch, a.scratch_pairs, [&](int o, float v) {
                    const int gi = g0 + o;
                    if (gi < a.dim) put(out + gi, L.bo ? __fadd_rn(v, __ldg(L.bo + gi)) : v, step);
                });
            }
            if (!(ok = wait_slots(ex + a.off_proj, a.dim, step, s.tmp, a))) break;   // C
            for (int i = tid; i < a.dim; i += nth) s.x[i] = __fadd_rn(s.x[i], s.tmp[i]);
            __syncthreads();
            if (tid == 0) put(ex + a.off_pres + cta, 0.0f, step);
            if (role.ffn0 < role.ffn1) {
                rmsnorm_exact(s.x, L.ffn_norm, a.dim, a.eps, s.xb, s.tmp, s.red);
                prepare(L.dt_up, s.xb, a.dim, s.prep);
                float *y = s.y;
                const int g0 = role.ffn0 * kTile;
                matvec_exact(L.dt_up, L.up, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, [&](int o, float v) {
                    const int gi = g0 + o;
                    y[o] = (L.b_up && gi < a.ffn) ? __fadd_rn(v, __ldg(L.b_up + gi)) : v;
                });
                if (L.dt_gate != L.dt_up) prepare(L.dt_gate, s.xb, a.dim, s.prep);
                uint64_t *out = ex + a.off_h;
                matvec_exact(L.dt_gate, L.gate, a.dim, role.ffn0, role.ffn1, s.prep, s.scratch, a.scratch_pairs, [&](int o, float g) {
                    const int gi = g0 + o;
                    if (gi < a.ffn) put(out + gi, silu_mul(y[o], g, a.elist, a.eindex), step);
                });
            }
            if (role.dn0 < role.dn1) {                                       // D
                if (!(ok = wait_slots(ex + a.off_h, a.ffn, step, s.xb, a))) break;
                prepare(L.dt_down, s.xb, a.ffn, s.prep);
                uint64_t *out = ex + a.off_down;
                const int g0 = role.dn0 * kTile;
                matvec_exact(L.dt_down, L.down, a.ffn, role.dn0, role.dn1, s.prep, s.scratch, a.scratch_pairs, [&](int o, float v) {
                    const int gi = g0 + o;
                    if (gi < a.dim) put(out + gi, L.b_down ? __fadd_rn(v, __ldg(L.b_down + gi)) : v, step);
                });
            }
        }
        if (!ok) break;
        {
            uint64_t *ex = a.ex + (step & 1) * a.ex_half;
            ok = wait_slots(ex + a.off_down, a.dim, step, s.tmp, a) && wait_slots(ex + a.off_pres, a.grid, step, nullptr, a);
            if (!ok) break;
            for (int i = tid; i < a.dim; i += nth) s.x[i] = __fadd_rn(s.x[i], s.tmp[i]);
            __syncthreads();
        }
        if (!last) continue;

        // Head: logits for this position and this CTA's share of the argmax.
        ++tcount;
        int host_stop = 0;
        if (cta == 0 && tid == 0) host_stop = ld_relaxed_sys_i32((const int *)&a.ctrl->stop_request);
        float best = -INFINITY;
        int best_i = -1;
        if (role.voc0 < role.voc1) {
            rmsnorm_exact(s.x, a.norm, a.dim, a.eps, s.xb, s.tmp, s.red);
            prepare(a.dt_head, s.xb, a.dim, s.prep);
            float *lg = a.logits + (size_t)pos * a.vocab;
            const int g0 = role.voc0 * kTile;
            matvec_exact(a.dt_head, a.head, a.dim, role.voc0, role.voc1, s.prep, s.scratch, a.scratch_pairs, [&](int o, float v) {
                const int gi = g0 + o;
                if (gi < a.vocab) {
                    lg[gi] = v;
                    if (v > best) { best = v; best_i = gi; }                  // this thread's outputs rise with o
                }
            });
        }
        if (stop_after) break;                                              // logits kept, nothing sampled
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
            if (mi < 0) mi = role.voc0 * kTile;                               // an empty or all-NaN slice
            uint64_t *tx = a.ex + (tcount & 1) * a.ex_half + a.off_tok + 3 * cta;
            put(tx, m, tcount);
            put(tx + 1, __int_as_float(mi), tcount);
            put(tx + 2, __int_as_float(host_stop), tcount);
        }
        __syncthreads();
        uint64_t *tx = a.ex + (tcount & 1) * a.ex_half + a.off_tok;
        if (!(ok = wait_slots(tx, 3 * a.grid, tcount, s.scores, a))) break;
        // Global argmax over the CTAs in vocabulary order (reference engine.c:299-300), same in every CTA.
        float gmax = -INFINITY;
        int next = 0;
        for (int c = 0; c < a.grid; c++) {
            if (s.scores[3 * c] > gmax) { gmax = s.scores[3 * c]; next = __float_as_int(s.scores[3 * c + 1]); }
        }
        const int stop_req = __float_as_int(s.scores[2]);
        __syncthreads();
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

extern "C" int l3m_decode_launch(const l3m::DecodeArgs *a, void *stream) {
    void *args[] = {(void *)a};
    cudaError_t e = cudaFuncSetAttribute(l3m::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, a->smem_bytes);
    if (e == cudaSuccess)
        e = cudaLaunchCooperativeKernel((const void *)l3m::decode_kernel, dim3(a->grid), dim3(512), args, (size_t)a->smem_bytes,
                                        (cudaStream_t)stream);
    if (e != cudaSuccess) {
        fprintf(stderr, "l3m: decode launch: %s\n", cudaGetErrorString(e));
        return -1;
    }
    return 0;
}

extern "C" int l3m_decode_occupancy(int smem_bytes) {
    int n = 0;
    if (cudaFuncSetAttribute(l3m::decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, l3m::decode_kernel, 512, smem_bytes) != cudaSuccess) return 0;
    return n;
}
