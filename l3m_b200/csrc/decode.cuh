// Shared host/device description of one GPU's decode state.
#pragma once
#include <cstdint>

namespace l3m {

struct alignas(16) LayerDev {
    const uint8_t *qkv;                 // rows: q of every head, then k of every kv head, then v
    const uint8_t *wo, *gate, *up, *down;   // gate NULL: up holds, per CTA, its up tiles then its gate tiles
    const float *attn_norm, *ffn_norm;
    const float *attn_norm_b, *ffn_norm_b;  // LayerNorm biases (NULL for RMSNorm files)
    const float *bq, *bk, *bv, *bo, *b_up, *b_down;   // NULL when absent
    uint16_t *kc, *vc;                  // K [n_kv][ctx][hd], V [n_kv][hd][vstride] bf16
    int dt_qkv, dt_wo, dt_gate, dt_up, dt_down;
    int st_qkv, st_wo, st_up, st_down;  // how many tiles of each fit in its part of the staging area
};

// One CTA's share of every phase (output tiles are 16 rows; ranges are [lo, hi)). Query heads
// head0, head0 + n_ctas, ... are this CTA's.
struct Role {
    int head0;
    int qkv0, qkv1, wo0, wo1, ffn0, ffn1, dn0, dn1, voc0, voc1;
};

// Host-mapped control block: tokens stream out, a stop request streams in.
struct Ctrl {
    volatile int32_t n_published;    // tokens written to tokens[]
    volatile int32_t done;           // 1 once the kernel has finished its loop
    volatile int32_t final_pos;      // last position run
    volatile int32_t n_gen;          // tokens the device accepted
    volatile int32_t stop_request;   // set by the host when on_token returns 0
    volatile int32_t error;          // nonzero: a device-side failure (kErr*)
    volatile int32_t where[4];       // the first failure: CTA, position, layer, wait (kWait*); for kErrShape
                                     // the launch shape seen: CTAs per cluster, clusters, grid, block
    volatile int32_t pad[2];
    // Launch statistics, written once when the loop ends: the exchange and token waits of the layer
    // cluster's CTAs (SM cycles, summed over its CTAs), the cold flushes' time (ns, excluded from token
    // time as the reference's --cold), and CTA 0's SM clock and global timer at the launch's start and
    // end (the cycles-to-time ratio of this launch).
    volatile unsigned long long wait_cyc, cold_ns, cyc0, cyc1, gt0, gt1;
};

constexpr int kDecodeThreads = 256;   // 8 warps per CTA
constexpr int kMaxShardGpus = 8;      // GPUs one model can be split over
constexpr int kClusterCtas = 16;      // one thread-block cluster runs the whole model
constexpr int kTraceEvents = 32;      // stamps per (position, layer); see the trace() calls in decode.cu

// The head phase runs on the helper clusters (and, in cold mode, on cluster 0 too): cluster 0 publishes
// x, every CTA with vocabulary tiles posts its (max, index), and CTA 0 reduces the posted slots. Waits
// are bounded by timeout_ns.
// The head's exchange between cluster 0 and the helper clusters, as self-validating 8-byte words (no
// flag, no count, no fence between data and signal): xw[i] = {tcount << 32 | bits of x[i]}, the
// final residual of the tcount-th sampled position, and xw[dim] = {tcount << 32 | position}, or
// kHeadDone as the position when generation ends; slots[c] = {head_epoch(tcount) << 56 | index << 32
// | bits of max}, CTA c's argmax (index < 2^24), written with a release so that the CTA's logits are
// visible first. The buffer is zeroed before every launch and tcount starts at 1, so no stale word
// carries a current epoch.
struct HeadX {
    unsigned long long *xw;             // [dim + 1]
    unsigned long long *slots;          // [grid]; posted by CTAs slot_lo.. only
    int *abort_flag;                    // [0]: first error code of any CTA; [1..4]: where (as Ctrl::where)
    unsigned long long *stats;          // [kClusterCtas]: each layer-cluster CTA's wait cycles at the end
    unsigned long long timeout_ns;
};
constexpr uint32_t kHeadDone = 0xFFFFFFFFu;
// The slot words' 8-bit epoch: 1..255, consecutive sampled positions always differ and none is 0.
__host__ __device__ inline uint32_t head_epoch(uint32_t tcount) { return 1u + (tcount - 1u) % 255u; }
// Error codes: a wait on another CTA gave up; a wait on a weight copy gave up; the launch does not
// have the shape the kernel was built for (cluster size, cluster count, grid, block); a sampled token
// outside the vocabulary.
enum { kErrNone = 0, kErrTimeout = 1, kErrStageTimeout = 2, kErrShape = 3, kErrToken = 4 };
// Which wait gave up (Ctrl::where[3]): exchanges 1-5 of a layer, the weight copy, the published x
// (helper clusters), the posted argmax slots (CTA 0).
enum { kWaitQkv = 1, kWaitAttn = 2, kWaitProj = 3, kWaitH = 4, kWaitDown = 5, kWaitStage = 8, kWaitHeadFlag = 9, kWaitHeadCount = 10,
       kWaitPeerAttn = 12, kWaitPeerProj = 13, kWaitPeerH = 14, kWaitPeerDown = 15, kWaitPeerToken = 16 };

// The vectors GPUs exchange each layer when a model is split over several (the reference's four
// all-gathers per layer, src/engine.c:254-274): attention output, wo output, gate output, down output.
enum { kXAttn = 0, kXProj = 1, kXH = 2, kXDown = 3, kXKinds = 4 };
// Forms of exchanges 2 and 4 (DecodeArgs::qx_attn, qx_h).
enum { kXFloat = 0, kXQ8 = 1, kXPrepF32 = 2, kXPrepBF16 = 3 };

// This GPU's share of an output-channel split over n_gpus GPUs (the reference's split over ranks,
// src/engine.c:467-476, at tile granularity, then over the CTAs of the GPU): query heads
// [head_lo, head_lo + n_heads_g) and kv heads [kv_lo, kv_lo + n_kv_g) (a kv head whose query heads
// straddle two GPUs is held by both, as src/engine.c:135-152), and the tile runs of wo and down
// (d_off..), up and gate (f_off..) and the head (v_off..). One GPU: the whole of everything.
struct Shard {
    int n_gpus, gpu;
    int head_lo, n_heads_g, kv_lo, n_kv_g, n_qkv_g;   // n_qkv_g = (n_heads_g + 2 n_kv_g) hd: this GPU's qkv rows
    int d_off, f_off, v_off;                           // first dim / ffn / vocab tile held
    int lo[kXKinds][kMaxShardGpus], len[kXKinds][kMaxShardGpus];   // every GPU's slice of each exchanged vector
    // n_gpus > 1: every GPU's receive buffers (peer-accessible device memory). rx[g][k]: 2 x the vector's
    // length of 8-byte words {value bits, epoch}, one half per layer parity; written by the GPUs that
    // produce the slices, polled by GPU g's CTAs. vote[g]: kMaxShardGpus words per sampled-position
    // parity {max bits, index | flags << 24} with the epoch in the second word. logits[g]: GPU g's logits
    // history. abort[g]: GPU g's abort word.
    unsigned long long *rx[kMaxShardGpus][kXKinds];
    unsigned long long *vote[kMaxShardGpus];
    float *logits[kMaxShardGpus];
    int *abort[kMaxShardGpus];
    uint32_t epoch0;                                   // the first epoch of this launch
    int all_logits;                                    // every GPU gets every logit (temperature sampling)
};

struct DecodeArgs {
    int dim, hd, ffn, vocab, ctx, n_heads, n_kv, hpk, n_layers, n_qkv, grid;   // n_qkv = (n_heads + 2 n_kv) hd; grid: all CTAs
    int slot_lo;                        // several clusters: the first CTA that posts a head slot (the
                                        // layer cluster posts none when the helpers take the whole head)
    HeadX hx;
    Shard sh;
    float eps;
    const LayerDev *layers;
    const uint8_t *head;
    int dt_head;
    const uint8_t *embed;
    int dt_embed;
    long long embed_row_bytes;
    const float *norm, *norm_b;         // final norm gain (and LayerNorm bias)
    int layernorm, gelu;                // GPT-2 family: LayerNorm instead of RMSNorm; GELU(up) instead of SiLU(gate) * up
    const float *pos_embed;             // [ctx][dim] learned positions (NULL: RoPE). Any of the three set: the
                                        // launch takes the kernel's GPT2 instance (only it reads them)
    const float2 *rope;                 // [ctx][hd/2] {cos, sin}
    const uint32_t *etab;               // libm expf exception set (hash table, expf_exact.h)
    const Role *roles;
    const int32_t *prompt;
    int n_prompt, max_new, eos, bos;
    float *logits;                      // [ctx][vocab]
    float temp;                         // > 0: sample (reference engine.c:370-384); else greedy
    unsigned long long rng;             // xorshift64* state, seeded as the reference (engine.c:555)
    float *probs;                       // [vocab] the sampling weights of the current position
    Ctrl *ctrl;
    int32_t *tokens;                    // host-mapped, ctx entries
    unsigned long long *trace;          // optional: [2][ctx][n_layers + 1][kTraceEvents] globaltimer stamps
    int trace_cta[2];
    // shared memory layout, byte offsets
    int sm_x, sm_xb, sm_tmp, sm_q8, sm_scale, sm_sum, sm_xf, sm_y, sm_scores, sm_kv, sm_att, sm_red, sm_kvbuf, sm_vt, sm_scratch;
    int sm_w_head;                      // a helper CTA's resident head tiles start here (it uses nothing after)
    int sm_wa, sm_wf, sm_wh, sm_rope;   // this layer's norm weights, the final norm, this position's RoPE row
    int sm_wab, sm_wfb, sm_whb;         // the same norms' LayerNorm biases
    int sm_layers;                      // a copy of layers[0 .. n_layers)
    int sm_xq, sm_xa, sm_xp, sm_xh, sm_xd, sm_xt;   // exchanged vectors: qkv, attn, proj, h, down; xt: the sampled token
                                                    // (next, stop, ok) and, one-cluster launch, each CTA c's slot at 4 + 4c
    // Weight staging area (the tiles of the next matvec phase, copied in by cp.async.bulk):
    // sm_w .. sm_w + w_bytes; its first w_extra bytes overlap the attention buffers (kvbuf, vt), so
    // the phases around attention (qkv, wo) use only [w_extra, w_bytes). sm_wbar: its mbarrier.
    int sm_w, w_bytes, w_extra, sm_wbar;
    int st_head;                        // head tiles that fit in the whole staging area (helper CTAs)
    // Exchanges 1-5 of a layer through st.async + per-CTA mbarriers (sm_xbar: 5 of them) instead of
    // cluster barriers; set when every CTA of the cluster produces qkv rows, which orders every
    // buffer's next write after all its reads (see decode.cu).
    int async_x, sm_xbar;
    // The form of exchanges 2 (attention output) and 4 (gate output), kX*: floats that phases B and D
    // prepare for wo / down; or, single-GPU with async exchanges, the activation already prepared by its
    // producer: q8 blocks with their scales and sums (the matrix quantised in every layer, every
    // producer's outputs whole blocks) stored into every CTA's sm_pa_* / sm_ph_*, or floats as the
    // matrix's prepare makes them (the same float dtype in every layer: bf16-rounded, or as they are)
    // stored into xa / xh. Either way phases B and D run no prepare.
    int qx_attn, qx_h;
    int sm_pa_q8, sm_pa_scale, sm_pa_sum, sm_ph_q8, sm_ph_scale, sm_ph_sum;
    int cold;                           // reference --cold (engine.c:330-338): before every position the layer cluster
                                        // streams cold_bytes (1.5 x L2) of scratch through its shared memory, evicting the
                                        // weights from L2 (timed apart); weight copies carry an L2 evict-first policy
    const uint8_t *cold_buf;
    unsigned long long cold_bytes;      // a multiple of kClusterCtas x cold_chunk
    int cold_chunk;                     // bytes per flush copy (a multiple of 16, at most w_extra)
    int vstride;                        // V cache: element i of position t at vc[i * vstride + t]
    int scratch_pairs, smem_bytes, attn_chunk;
};

}  // namespace l3m
