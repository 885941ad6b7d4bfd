// Shared host/device description of one GPU's decode state.
#pragma once
#include <cstdint>

namespace l3m {

struct LayerDev {
    const uint8_t *qkv;                 // one unit per query head: its q rows, then its kv head's k and v rows
    const uint8_t *wo, *gate, *up, *down;
    const float *attn_norm, *ffn_norm;
    const float *bq, *bk, *bv, *bo, *b_up, *b_down;   // NULL when absent
    uint16_t *kc, *vc;                  // [n_kv][ctx][hd] bf16
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
    uint64_t *ex;                       // exchange slots: two halves by parity
    long long ex_half;                  // slots per half
    int off_attn, off_proj, off_h, off_down, off_pres, off_tok;
    const int32_t *prompt;
    int n_prompt, max_new, eos, bos;
    float *logits;                      // [ctx][vocab]
    Ctrl *ctrl;
    int32_t *tokens;                    // host-mapped, ctx entries
    int *abort_flag;                    // device: first error code
    unsigned long long timeout_ns;      // per wait
    // shared memory layout, byte offsets
    int sm_x, sm_xb, sm_tmp, sm_q8, sm_scale, sm_sum, sm_xf, sm_y, sm_scores, sm_kv, sm_att, sm_red, sm_scratch;
    int scratch_pairs, smem_bytes;
};

}  // namespace l3m
