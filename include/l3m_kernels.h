// l3m matvec entry points, B200 build. The host-pointer table keeps the reference's kernel-table
// shape (fpedd/l3m src/kernels.h:24-52) so its kernel tests drive the GPU kernels unchanged; the
// *_dev entry points take device pointers and a CUDA stream (passed as void *) and return 0 or a
// negative error (message from l3m_cuda_error()). No CUDA or torch types appear in any signature.
//
// Tile layout (the reference's, src/kernels.h:1-10, byte for byte): L3M_TILE = 16 outputs x K inputs,
//   f32   [K][16] float
//   bf16  [K/2][16][2] bf16
//   q8_0  per 32 inputs: d[16] f16, q[8][16][4] u8 = value + 128                 544 bytes
//   q4_0  per 32 inputs: d[16] f16, q[4][16][4] nibbles, value = nibble - 8     288 bytes
//   mxfp4 per 32 inputs: e[16] e8m0, the same nibbles, value = LUT[nibble]       272 bytes
// Each 64-byte line holds one 4-byte group of all 16 outputs, so a warp's 16-byte loads of a
// block are fully coalesced and every block starts 16-byte aligned.
#pragma once
#include <stddef.h>
#include <stdint.h>

#define L3M_API __attribute__((visibility("default")))
#define L3M_TILE   16
#define L3M_QBLOCK 32

#ifdef __cplusplus
extern "C" {
#endif

enum { L3M_DT_F32, L3M_DT_BF16, L3M_DT_Q8_0, L3M_DT_Q4_0, L3M_DT_MXFP4, L3M_DT_COUNT };

// The prepared activation (reference src/kernels.h:24-30): bf16 copy, or q8 with a per-32 scale and sum.
typedef struct {
    const float    *f32;
    const uint16_t *bf16;
    const int8_t   *q8;     // x[i] ~= q8[i] * scale[i/32]
    const float    *scale;  // n/32 entries
    const int32_t  *sum;    // n/32 entries: sum of q8 over the block
} l3m_vec;

// y[0 .. ntiles*16) = tiles . x, all host pointers (reference src/kernels.h:33). The GPU tables copy
// in, launch on the current device and copy out: a test and drop-in shim, not the fast path.
typedef void (*l3m_gemv_fn)(float *y, const void *tiles, int ntiles, int k, const l3m_vec *x);

typedef struct {                                   // reference src/kernels.h:35-40
    const char *name;
    l3m_gemv_fn gemv[L3M_DT_COUNT];
    void (*attend)(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int head_dim, int stride);
} l3m_kernels;

// "sm100a": results bit-identical to the reference's scalar table (src/kernels_scalar.c) for every
// dtype. "sm100a-fast": quantised dtypes identical as well; f32 and bf16 reassociate the sum over
// K across threads (tolerance-checked, like the reference's AVX tables).
L3M_API extern const l3m_kernels l3m_kernels_sm100a, l3m_kernels_sm100a_fast;

// Replaces reference src/dispatch.c:28-36: L3M_ISA=sm100a|sm100a-fast selects a table; anything else
// is reported and the default (sm100a) is used. There is no CPU table: without a usable B200 the
// engine's load fails with a message.
L3M_API const l3m_kernels *l3m_kernels_pick(void);
L3M_API int                l3m_kernels_usable(const l3m_kernels *k);   // 1 when a CUDA device of compute capability 10.x is present

// Layout helpers (reference src/kernels.h:48-52), host code.
L3M_API size_t l3m_row_bytes(int dtype, int k);
L3M_API size_t l3m_tile_bytes(int dtype, int k);
L3M_API void   l3m_pack_tile(void *dst, int dtype, const void *const rows[L3M_TILE], int k);   // NULL row = zeros
L3M_API void   l3m_dequant_row(float *out, int dtype, const void *row, int k);
L3M_API void   l3m_vec_prepare(l3m_vec *v, int dtype, const float *x, int n, void *scratch);    // scratch >= 2n + n/4 bytes

// ---- device entry points (no counterpart in the reference: the GPU-resident forms of the above)

// y = tiles . x on the device. exact bit 0: 1 the sm100a table's order, 0 sm100a-fast. exact bit 1
// (L3M_GEMV_CONST_TILES): the caller guarantees that no work issued earlier on the stream writes the
// tiles (model weights), so the streamed kernel may start reading them before that work has finished
// (x and y keep the stream order); successive calls then overlap.
#define L3M_GEMV_CONST_TILES 2
L3M_API int l3m_gemv_dev(int exact, int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream);
// The exact quantised matvec (the same y as l3m_gemv_dev with exact = 1, bit for bit) for callers
// that must not allocate device memory, such as a host whose framework owns the device's memory
// pool, or a decode loop where the implicit device synchronisation of cudaMalloc/cudaFree would
// stall other streams. No counterpart in the reference. K is split across every SM through one
// fixed 4 MiB device buffer inside this library: q8_0/q4_0/mxfp4 only, at most 524,288 block
// results per call (ntiles*16*k/32), larger calls return -1 and launch nothing. The buffer is
// shared by all calls on a device, so overlapping calls (two streams or threads) race and must be
// serialised. The first call on each device looks the buffer's address up and keeps it for the
// process's life, so do not reset a device this entry has used.
// Pointers must be 4-byte aligned (refused with -1 otherwise).
L3M_API int l3m_gemv_splitk_dev(int dtype, float *y, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream);
// One draw of the reference's temperature sampler (src/engine.c:98-101, 283-287, 370-384, one
// rank) over logits[0..vocab) on the device: weights expf((l - max) / temperature) (0 below -16),
// the first index whose running double sum exceeds u * (the whole sum), u the next xorshift64*
// draw of *rng_state (advanced); the last index when none does. rng_state, token: device memory;
// scratch: vocab floats of device memory. temperature must be > 0. Tests use it; l3m_generate
// samples inside its own kernel with the same code.
L3M_API int l3m_sample_dev(const float *logits, int vocab, float temperature, uint64_t *rng_state, int32_t *token, float *scratch,
                           void *stream);
// Prepare x[0..n) for dtype on the device, as l3m_vec_prepare. scratch (device) >= 2n + n/4 bytes.
L3M_API int l3m_vec_prepare_dev(int dtype, l3m_vec *out, const float *x, int n, void *scratch, void *stream);
// The exact integer part of each quantised kernel: dots[(t*16 + c)*(k/32) + b] = sum_i w*q8_x over block b
// of output c in tile t, the dtype's offset already removed (the value the epilogue converts to float).
L3M_API int l3m_block_dots_dev(int dtype, int32_t *dots, const void *tiles, int ntiles, int k, const l3m_vec *x, void *stream);
// Unpack quantised tiles on the device: integer weights q[(t*16+c)*k + i] and block scales d[(t*16+c)*(k/32) + b].
L3M_API int l3m_unpack_dev(int dtype, int8_t *q, float *d, const void *tiles, int ntiles, int k, void *stream);
// One head of causal attention over a bf16 KV cache (reference src/ops.h:14-16), device pointers.
L3M_API int l3m_attend_dev(float *out, const float *q, const uint16_t *k, const uint16_t *v, int pos, int head_dim, int stride, void *stream);
// y[i] = expf(x[i]) for i < n on the device, bit for bit the host C library's expf (the function the
// reference's softmax, SiLU and sampler call, src/ops.c:45, 50; the kernels above use the same code).
// x, y: device memory.
L3M_API int l3m_expf_dev(const float *x, float *y, int n, void *stream);
// Diagnostics: the SM cycles per step of a dependent fp32 fma chain (operands in registers), timed
// on the current device over `steps` steps (64 .. 2^24) by one warp; synchronous. The decode's
// chain-latency bound is its dependent steps per token times this.
L3M_API int l3m_chain_cycles_dev(int steps, double *cycles_per_step);
// The last CUDA error this library saw, as text ("" if none).
L3M_API const char *l3m_cuda_error(void);

#ifdef __cplusplus
}
#endif
