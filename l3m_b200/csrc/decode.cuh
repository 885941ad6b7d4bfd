// Shared host/device description of one GPU's decode state.
#pragma once
#include <cstdint>

namespace l3m {

struct alignas(16) LayerDev {
    const uint8_t *qkv;                 // one unit per query head: its q rows, then its kv head's k and v rows
    const uint8_t *wo, *gate, *up, *down;
    const float *attn_norm, *ffn_norm;
    const float *bq, *bk, *bv, *bo, *b_up, *b_down;   // NULL when absent
    uint16_t *kc, *vc;                  // K [n_kv][ctx][hd], V [n_kv][hd][vstride] bf16
    int dt_qkv, dt_wo, dt_gate, dt_up, dt_down;
};

// One CTA's share of every phase (output tiles are 16 rows; ranges are [lo, hi)).
struct Role {
    int head;          // query head of the attention phase, -1 for none
    int kv_writer;     // 1: stores the KV row of its kv head
    int wo0, wo1, ffn0, ffn1, dn0, dn1, voc0, voc1;
};

// Host-mapped control block: tokens stream out, a stop request streams in.
struct Ctrl {
    volatile int32_t n_published;    // tokens written to tokens[]
    volatile int32_t done;           // 1 once the kernel has finished its loop
    volatile int32_t final_pos;      // last position run
    volatile int32_t n_gen;          // tokens the device accepted
    volatile int32_t stop_request;   // set by the host when on_token returns 0
    volatile int32_t error;          // nonzero: see kErr*
    volatile int32_t pad[2];
};

enum { kErrNone = 0, kErrTimeout = 1, kErrEpoch = 2 };
constexpr int kDecodeThreads = 256;   // 8 warps: the register file holds every live value without spilling

// Exchanges between phases. Each has a float data buffer and an arrival counter, both in two halves
// by step parity. A producer writes its outputs and adds 1 (release) to the counter; a consumer's
// thread 0 polls the counter (acquire) until every expected arrival of this step is in, then the CTA
// reads the data once. Counters sit on their own 128-byte lines.
enum { kXAttn, kXProj, kXH, kXDown, kXTok, kXCount };

struct DecodeArgs {
    int dim, hd, ffn, vocab, ctx, n_heads, n_kv, hpk, n_layers, unit_tiles, grid;
    float eps;
    const LayerDev *layers;
    const uint8_t *head;
    int dt_head;
    const uint8_t *embed;
    int dt_embed;
    long long embed_row_bytes;
    const float *norm;
    const float2 *rope;                 // [ctx][hd/2] {cos, sin}; NULL: learned positions
    const uint32_t *elist, *eindex;     // libm expf exception list
    const Role *roles;
    float *xd;                          // exchange data, two halves of xd_half floats
    long long xd_half;
    int d_attn, d_proj, d_h, d_down, d_tok;   // float offsets within a half
    uint32_t *ctr;                      // [kXCount][2] counters, 32 words apart
    int arrivals[kXCount];              // per use: producers (+ every CTA's presence for kXDown)
    const int32_t *prompt;
    int n_prompt, max_new, eos, bos;
    float *logits;                      // [ctx][vocab]
    Ctrl *ctrl;
    int32_t *tokens;                    // host-mapped, ctx entries
    int *abort_flag;                    // device: first error code
    unsigned long long timeout_ns;      // per wait
    unsigned long long *trace;          // optional: [4][ctx][n_layers + 1][16] globaltimer stamps
    int trace_cta[4];
    // shared memory layout, byte offsets
    int sm_x, sm_xb, sm_tmp, sm_q8, sm_scale, sm_sum, sm_xf, sm_y, sm_y2, sm_scores, sm_kv, sm_att, sm_red, sm_kvbuf, sm_vt, sm_scratch;
    int sm_wa, sm_wf, sm_wh, sm_rope;   // this layer's norm weights, the final norm, this position's RoPE row
    int sm_layers;                      // a copy of layers[0 .. n_layers)
    int vstride;                        // V cache: element i of position t at vc[i * vstride + t]
    int scratch_pairs, smem_bytes, attn_chunk;
};

}  // namespace l3m
