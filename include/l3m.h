// l3m public C API, B200 build: load a model onto one or more GPUs, generate, tokenize, read the
// counters. Every declaration keeps the reference's signature and contract (fpedd/l3m src/l3m.h:6-58)
// so existing callers (its ctypes binding python/l3m/__init__.py:30-50, its CLI src/main.c, its
// tests) work unchanged; the few reinterpretations for GPUs are stated beside each field.
#pragma once
#include <stdint.h>
#include <stdio.h>

#define L3M_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

typedef struct l3m_model l3m_model;

// Field order and types are the reference's (src/l3m.h:10-19): the struct is ABI.
typedef struct {
    const int *cpus;       // GPU ordinals to shard over, in rank order; NULL = GPU 0 alone
    int        n_cpus;     // number of GPUs in cpus
    int        ctx;        // KV cache length, 0 = min(model context, 512)
    int        reference;  // 1 = the fp32 reference path (no activation quantisation), on the GPU
    int        force;      // 1 = load even if the weights will not stay resident in the persisting L2 window
    int        verbose;    // print each GPU's shard sizes against its L2 budget, on stderr
    int        cold;       // 1 = the weights are evicted from L2 before every position (time excluded), no persisting window
} l3m_opts;

// Field order and types are the reference's (src/l3m.h:21-29).
typedef struct {
    double tokens;         // forward passes since the previous read, prompt included
    double ns_token;       // wall time per token
    double ns_compute;     // per token, ns_token - ns_wait
    double ns_wait;        // per token, time the layer cluster's CTAs spend in exchange and token waits (their average)
    double bytes_token;    // weight bytes streamed per token, summed over the GPUs (padding included)
    double l2_bytes;       // L2 cache summed over the GPUs
    double l3_miss, dram_bytes, energy_j, llc_occupancy;   // NAN: CPU counters, not measured on GPUs
} l3m_perf;

// opts may be NULL. Returns NULL on failure, with the reason on stderr ("l3m: ...").
L3M_API l3m_model   *l3m_load(const char *path, const l3m_opts *opts);
L3M_API void         l3m_free(l3m_model *m);

// Feed the prompt, then sample up to max_new tokens, stopping early at EOS, BOS or the end of the
// context. on_token (may be NULL) is called on the caller's thread with each new token, never the
// prompt, EOS or BOS, and stops generation by returning 0. Returns the number of tokens generated,
// 0 if the prompt is empty or does not fit in ctx, -1 if a prompt id is outside [0, vocab) or the
// GPU reported an error. temperature 0 = greedy. Calls on one model must not overlap, nor come
// from on_token.
L3M_API int          l3m_generate(l3m_model *m, const int32_t *prompt, int n_prompt, int max_new,
                                  float temperature, uint64_t seed, int (*on_token)(int32_t tok, void *user), void *user);
L3M_API const float *l3m_logits(const l3m_model *m);   // vocab floats: the prediction after the last token fed
L3M_API int          l3m_vocab(const l3m_model *m);
L3M_API int          l3m_ctx(const l3m_model *m);
L3M_API const char  *l3m_describe(const l3m_model *m);  // "<file>: <dtype>, <n> layers, <size> MiB on <n> GPU(s) (<table>)"

L3M_API int          l3m_encode(const l3m_model *m, const char *text, int add_bos, int32_t *out, int max);
L3M_API const char  *l3m_decode(const l3m_model *m, int32_t tok, int *len);   // raw bytes, not NUL-terminated
L3M_API int          l3m_bos(const l3m_model *m);   // -1 if the model has none
L3M_API int          l3m_eos(const l3m_model *m);
L3M_API const char  *l3m_chatml(const l3m_model *m, int32_t *im_start);

L3M_API int          l3m_perf_read(l3m_model *m, l3m_perf *out);   // since the previous read; -1 if nothing ran
// Extension (not in the reference's API): device time of the decode launches since the previous
// l3m_perf_read (CUDA events around each launch, cold flushes excluded), ns.
L3M_API double       l3m_device_ns(const l3m_model *m);

L3M_API int          l3m_parse_cpus(const char *list, int *cpus, int max);   // "0-7,12" -> count, -1 on error
L3M_API void         l3m_print_hw(FILE *out);                        // the GPUs, their L2 and persisting budgets

// No counterpart in the reference: copy the .l3m file `in` to `out` with a packed section appended
// (every matrix the GPU streams, already in its tile order, as extra tensors named "b200v1.*" that a
// v1 reader ignores), so that l3m_load copies those bytes instead of repacking rows. Host only (no
// GPU); 0 on success, -1 with the reason on stderr.
L3M_API int          l3m_write_packed(const char *in, const char *out);

#ifdef __cplusplus
}
#endif
