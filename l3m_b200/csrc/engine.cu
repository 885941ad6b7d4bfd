// The B200 decode engine behind include/l3m.h. Replaces the reference's sharded CPU engine
// (src/engine.c:1-603) with a device-resident one:
//   load      validate the file, pack every matrix into 16-output tiles in one device arena (the
//             streamed weights first, so one persisting-L2 window covers them), give each CTA its
//             share of every phase, refuse when the weights exceed the L2 persisting budget unless
//             forced (the reference's cache-budget refusal, src/engine.c:496-525);
//   generate  one launch of the decode kernel (a single thread-block cluster) per call; tokens stream back
//             through host-mapped memory to on_token on the caller's thread, and a stop request
//             streams in the other way.
#include <cuda_runtime.h>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <deque>
#include <string>
#include <vector>
#include <x86intrin.h>
#include "file.h"
#include "numerics.h"
#include "ops.cuh"
#include "decode.cuh"
#include "../../include/l3m.h"
#include "../../include/l3m_kernels.h"

extern "C" int l3m_decode_launch(const l3m::DecodeArgs *a, const l3m::DecodeArgs *a_dev, void *stream);
extern "C" int l3m_decode_occupancy(int smem_bytes);
extern "C" int l3m_decode_smem_budget(void);
extern "C" int l3m_expf_table(const uint32_t **table);

namespace {

constexpr int kMaxGpus = 8;
constexpr int kDefaultCtx = 512;
constexpr double MiB = 1024.0 * 1024.0;

double now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e9 + ts.tv_nsec;
}

int tiles_of(int n) { return (n + L3M_TILE - 1) / L3M_TILE; }

struct Gpu {
    int dev = -1, sms = 0, rank = 0;
    cudaStream_t stream = nullptr, side = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    uint8_t *arena = nullptr;
    size_t arena_bytes = 0, weight_bytes = 0, held_bytes = 0;
    uint16_t *kv = nullptr;
    size_t kv_bytes = 0;
    float2 *rope = nullptr;
    l3m::LayerDev *layers = nullptr;
    l3m::Role *roles = nullptr;
    l3m::DecodeArgs *args_dev = nullptr;
    unsigned long long *trace = nullptr;
    size_t trace_bytes = 0;
    void *hx = nullptr;
    size_t hx_bytes = 0;
    int32_t *prompt = nullptr;
    float *logits = nullptr;
    float *probs = nullptr;                                            // [vocab] sampling weights
    unsigned long long *rx = nullptr, *vote = nullptr;                 // receive buffers and votes from other GPUs
    size_t rx_bytes = 0, vote_bytes = 0;
    uint8_t *cold = nullptr;                                           // cold mode: the scratch streamed before each position
    l3m::DecodeArgs args{};
    size_t l2_bytes = 0, persist_max = 0, window_max = 0, prev_limit = 0;
    bool limit_set = false;
    std::string name;
};

}  // namespace

struct l3m_model {
    l3m_file f;
    int n_gpus = 0;
    Gpu g[kMaxGpus];
    int dim = 0, hd = 0, ffn = 0, vocab = 0, ctx = 0, n_heads = 0, n_kv = 0, hpk = 0, n_layers = 0;
    unsigned flags = 0;
    int reference = 0, cold = 0;
    l3m::Ctrl *ctrl = nullptr;                                         // one per GPU, host-mapped; GPU 0 streams the tokens
    int32_t *tokens = nullptr;
    l3m::Ctrl *ctrl_dev = nullptr;
    uint32_t epoch_next = 1;                                           // the next launch's first exchange epoch
    int32_t *tokens_dev = nullptr;
    std::vector<float> host_logits;
    int logits_pos = -1, cached_pos = -2;
    double tok_count = 0, ns = 0, dev_ns = 0, wait_ns = 0, cold_ns = 0;   // since the last l3m_perf_read
    size_t weight_bytes = 0;
    const l3m_kernels *kk = nullptr;
    char desc[256] = {0};
};

namespace {

l3m_model *fail(l3m_model *m, const char *msg) {
    fprintf(stderr, "l3m: %s\n", msg);
    l3m_free(m);
    return nullptr;
}

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    fprintf(stderr, "l3m: %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

// Host staging of one GPU's arena; every part starts 256-byte aligned.
struct Stage {
    std::vector<uint8_t> buf;
    size_t put(const void *src, size_t n) {
        size_t off = (buf.size() + 255) & ~(size_t)255;
        buf.resize(off + n);
        if (src) memcpy(buf.data() + off, src, n);
        return off;
    }
    size_t reserve(size_t n) { return put(nullptr, n); }
};

const void *row_ptr(const l3m_file *f, const l3m_tensor *t, int r) {
    return (const uint8_t *)l3m_file_data(f, t) + (size_t)r * l3m_row_bytes((int)t->dtype, (int)t->shape[1]);
}

// Rows of one matrix to pack, as file rows (dtype of the tensor) or, on the reference path,
// dequantised f32 copies (the fp32 reference dequantises every matrix, src/ref.c:24-32). A NULL
// row packs as zeros.
struct Rows {
    int dtype = 0, k = 0;
    std::vector<const void *> ptr;
    std::deque<std::vector<float>> f32;          // stable addresses as it grows
    void add(const l3m_file *f, const l3m_tensor *t, int r, bool to_f32) {
        k = (int)t->shape[1];
        if (!to_f32) {
            dtype = (int)t->dtype;
            ptr.push_back(row_ptr(f, t, r));
            return;
        }
        dtype = L3M_F32;
        f32.emplace_back(k);
        l3m_dequant_row(f32.back().data(), (int)t->dtype, row_ptr(f, t, r), k);
        ptr.push_back(f32.back().data());
    }
};

size_t pack(Stage &s, Rows &rows) {
    const int n = (int)rows.ptr.size(), nt = tiles_of(n);
    const size_t tb = l3m_tile_bytes(rows.dtype, rows.k);
    size_t off = s.reserve((size_t)nt * tb);
    for (int t = 0; t < nt; t++) {
        const void *tr[L3M_TILE];
        for (int j = 0; j < L3M_TILE; j++) tr[j] = t * L3M_TILE + j < n ? rows.ptr[t * L3M_TILE + j] : nullptr;
        l3m_pack_tile(s.buf.data() + off + (size_t)t * tb, rows.dtype, tr, rows.k);
    }
    return off;
}

// RoPE coefficients with the reference's exact expressions and this host's libm (src/ops.c:29-33).
std::vector<float2> rope_table(int ctx, int hd, float theta) {
    std::vector<float2> t((size_t)ctx * (hd / 2));
    for (int pos = 0; pos < ctx; pos++)
        for (int i = 0; i < hd / 2; i++) {
            volatile float e = -2.0f * (float)i / (float)hd;
            float angle = (float)pos * powf(theta, e);
            t[(size_t)pos * (hd / 2) + i] = make_float2(cosf(angle), sinf(angle));
        }
    return t;
}

void split(int n, int parts, int r, int *lo, int *hi) {   // reference src/engine.c:88-91
    *lo = (int)((long)n * r / parts);
    *hi = (int)((long)n * (r + 1) / parts);
}

int align16(int x) { return (x + 15) & ~15; }

// The matrices the decode kernel streams, packed into 16-row tiles in the order and grouping the
// kernel reads them: per layer the flat q|k|v rows, wo, up and gate (one matrix holding, per CTA of
// the cluster, its up tiles then its gate tiles, when they share a dtype; up alone for a GELU MLP),
// down; then the head. A file may carry any of them already packed ("b200v1." + the name below,
// written by l3m_write_packed): those bytes are copied instead of packed from rows.
struct Streamed {
    std::vector<size_t> off_qkv, off_wo, off_up, off_gate, off_down;   // off_gate (size_t)-1: none (in up, or GELU)
    std::vector<int> dt_qkv, dt_wo, dt_up, dt_gate, dt_down;
    size_t off_head = 0;
    int dt_head = 0;
    struct Entry { std::string name; size_t off, rows; int dtype, k; };
    std::vector<Entry> entries;                  // every packed matrix, for the writer
    size_t widened = 0;                          // bytes added by widening q4_0 / mxfp4 matrices to q8_0
};
constexpr const char *kPackedPrefix = "b200v1.";

// q4_0 and mxfp4 tiles rewritten as q8_0 tiles with the same block dots and scales, so the decode
// kernel multiplies them with q8_0's one dp4a per 4 inputs instead of unpacking nibbles. A q8_0 byte
// is the weight + 128 (offset 128): a q4_0 code c (the reference's dot uses c with offset 8) becomes
// c + 120, and an mxfp4 code's doubled e2m1 value v (offset 16 on v + 16) becomes v + 128, so
// sum(byte * x) - 128 * sum(x) is the reference's integer dot exactly. Scales: q4_0's f16 as they
// are; mxfp4's 2^(e - 128) as the f16 holding exactly that value, which exists for e in [104, 143]
// (mxfp4_fits checks a matrix first). Source block: scales, then byte j of group g of row c at
// (g*16 + c)*4 + j holding inputs 8g+j (low nibble) and 8g+4+j (high nibble); q8_0 block: 16 f16
// scales, then input i of row c at (i/4*16 + c)*4 + i%4 (reference src/pack.c).
bool mxfp4_fits(const uint8_t *src, size_t ntiles, int k) {
    const size_t blocks = ntiles * (size_t)(k / L3M_QBLOCK);
    for (size_t b = 0; b < blocks; b++)
        for (int c = 0; c < L3M_TILE; c++) {
            const int e = src[b * 272 + c];
            if (e < 104 || e > 143) return false;
        }
    return true;
}
void widen_to_q8(int dtype, const uint8_t *src, uint8_t *dst, size_t ntiles, int k) {
    const int sb = dtype == L3M_MXFP4 ? 16 : 32, in_b = sb + 256;
    uint8_t val[16];
    for (int n = 0; n < 16; n++) val[n] = (uint8_t)(dtype == L3M_MXFP4 ? l3m_mxfp4_value(n) + 128 : n + 120);
    for (size_t b = 0; b < ntiles * (size_t)(k / L3M_QBLOCK); b++) {
        const uint8_t *in = src + b * in_b;
        uint8_t *out = dst + b * 544;
        if (dtype == L3M_MXFP4) {
            for (int c = 0; c < L3M_TILE; c++) {                               // 2^p, p = e - 128 in [-24, 15]
                const int p = (int)in[c] - 128;
                const uint16_t h = (uint16_t)(p >= -14 ? (p + 15) << 10 : 1 << (p + 24));
                memcpy(out + 2 * c, &h, 2);
            }
        } else {
            memcpy(out, in, 32);
        }
        uint8_t *w = out + 32;
        for (int g = 0; g < 4; g++)
            for (int c = 0; c < L3M_TILE; c++)
                for (int j = 0; j < 4; j++) {
                    const uint8_t v = in[sb + (g * L3M_TILE + c) * 4 + j];
                    const int i0 = 8 * g + j, i1 = 8 * g + 4 + j;
                    w[(i0 / 4 * L3M_TILE + c) * 4 + i0 % 4] = val[v & 15];
                    w[(i1 / 4 * L3M_TILE + c) * 4 + i1 % 4] = val[v >> 4];
                }
    }
}

// Which q4_0 / mxfp4 matrices the decode kernel gets as q8_0 tiles: only where a CTA's whole share of
// the widened tiles fits the part of the staging area that matrix is copied into (else the kernel
// would read the rest from global memory, slower than unpacking nibbles from shared memory).
struct Widen {
    bool on = false;
    long cap_qkv_wo = 0, cap_rest = 0;   // staging bytes for qkv / wo, and for up(+gate) / down
    long cap_head = 0;                   // a helper CTA's resident head tiles
    int head_ctas = 1;                   // the CTAs the head's tiles are split over
};

// widen: q4_0 and mxfp4 matrices go to the device as q8_0 tiles (widen_to_q8; an mxfp4 matrix only
// when every scale has an f16 form) when per_cta tiles of them fit in cap bytes; *dtype is then
// L3M_Q8_0 and out.widened counts the extra bytes. The writer's entries keep the file's layout.
size_t pack_rows(Stage &s, Rows &r, const l3m_file *f, const std::string &name, Streamed &out, bool ref, const Widen &wd, long cap,
                 int per_cta, int *dtype) {
    const bool widen = wd.on && (long)per_cta * (r.k / L3M_QBLOCK) * (long)l3m_tile_bytes(L3M_Q8_0, L3M_QBLOCK) <= cap;
    const size_t rows = (size_t)tiles_of((int)r.ptr.size()) * L3M_TILE, tb = l3m_tile_bytes(r.dtype, r.k);
    *dtype = r.dtype;
    const l3m_tensor *pt = ref ? nullptr : l3m_file_tensor(f, (kPackedPrefix + name).c_str());
    size_t off;
    if (pt && (int)pt->dtype == r.dtype && pt->ndim == 2 && pt->shape[0] == rows && (int)pt->shape[1] == r.k && pt->nbytes == rows / L3M_TILE * tb)
        off = s.put(l3m_file_data(f, pt), (size_t)pt->nbytes);
    else
        off = pack(s, r);
    out.entries.push_back({name, off, rows, r.dtype, r.k});
    const size_t nt = rows / L3M_TILE;
    if (widen && rows && (r.dtype == L3M_Q4_0 || (r.dtype == L3M_MXFP4 && mxfp4_fits(s.buf.data() + off, nt, r.k)))) {
        const size_t bytes = nt * tb, wide = nt * l3m_tile_bytes(L3M_Q8_0, r.k);
        const std::vector<uint8_t> packed(s.buf.begin() + off, s.buf.begin() + off + bytes);
        s.buf.resize(off);                                                          // the packed copy was the last put
        off = s.reserve(wide);
        widen_to_q8(r.dtype, packed.data(), s.buf.data() + off, nt, r.k);
        out.widened += wide - bytes;
        *dtype = L3M_Q8_0;
    }
    return off;
}

// The rows one GPU holds of an output-channel split over n GPUs (the reference's split over ranks,
// src/engine.c:467-476, with the kv heads of src/engine.c:135-152; vocabulary tiles split evenly, as
// the reference's greedy deal comes out with equal budgets): query heads [head_lo, head_hi), kv heads
// [kv_lo, kv_hi), and tile runs of the dim (wo, down), ffn (up, gate) and vocabulary (head) rows.
struct ShardRange {
    int head_lo, head_hi, kv_lo, kv_hi, d_lo, d_hi, f_lo, f_hi, v_lo, v_hi;
    bool whole;                                                   // one GPU: the packed section of the file applies
};

ShardRange shard_range(const l3m_header *h, int n, int r) {
    ShardRange s;
    const int hpk = (int)(h->n_heads / h->n_kv_heads);
    split((int)h->n_heads, n, r, &s.head_lo, &s.head_hi);
    s.kv_lo = s.head_lo / hpk;
    s.kv_hi = s.head_hi > s.head_lo ? (s.head_hi - 1) / hpk + 1 : s.kv_lo;
    split(tiles_of((int)h->dim), n, r, &s.d_lo, &s.d_hi);
    split(tiles_of((int)h->ffn_dim), n, r, &s.f_lo, &s.f_hi);
    split(tiles_of((int)h->vocab), n, r, &s.v_lo, &s.v_hi);
    s.whole = n == 1;
    return s;
}

// Rows [lo, hi) of t that exist (rows past the matrix pack as zeros).
void add_rows(Rows &r, const l3m_file *f, const l3m_tensor *t, int lo, int hi, bool ref) {
    for (int i = lo; i < hi; i++) {
        if (i < (int)t->shape[0]) r.add(f, t, i, ref);
        else r.ptr.push_back(nullptr);
    }
}

void pack_streamed(const l3m_file *f, bool ref, const ShardRange &sr, int hd, Stage &s, Streamed &out, const Widen &wide = Widen{}) {
    const int L = (int)f->h->n_layers;
    const bool packed_ok = sr.whole && !ref;                                        // the file's b200v1 section is for one GPU
    for (auto *v : {&out.off_qkv, &out.off_wo, &out.off_up, &out.off_gate, &out.off_down}) v->assign(L, 0);
    for (auto *v : {&out.dt_qkv, &out.dt_wo, &out.dt_up, &out.dt_gate, &out.dt_down}) v->assign(L, 0);
    const int T = L3M_TILE, ftiles = sr.f_hi - sr.f_lo;
    auto share = [](int tiles) { return (tiles + l3m::kClusterCtas - 1) / l3m::kClusterCtas; };   // a layer CTA's largest share
    for (int l = 0; l < L; l++) {
        const std::string b = "blk." + std::to_string(l) + ".";
        const l3m_tensor *wq = l3m_file_blk(f, l, "wq"), *wk = l3m_file_blk(f, l, "wk"), *wv = l3m_file_blk(f, l, "wv");
        Rows r;                                                                     // q of the heads, then k, then v
        add_rows(r, f, wq, sr.head_lo * hd, sr.head_hi * hd, ref);
        add_rows(r, f, wk, sr.kv_lo * hd, sr.kv_hi * hd, ref);
        add_rows(r, f, wv, sr.kv_lo * hd, sr.kv_hi * hd, ref);
        if (r.ptr.empty()) r.k = (int)wq->shape[1], r.dtype = ref ? L3M_F32 : (int)wq->dtype;
        out.off_qkv[l] = pack_rows(s, r, f, b + "qkv", out, !packed_ok, wide, wide.cap_qkv_wo, share(tiles_of((int)r.ptr.size())), &out.dt_qkv[l]);
        {
            Rows ro;
            const l3m_tensor *wo = l3m_file_blk(f, l, "wo");
            add_rows(ro, f, wo, sr.d_lo * T, std::min(sr.d_hi * T, (int)wo->shape[0]), ref);
            out.off_wo[l] = pack_rows(s, ro, f, b + "wo", out, !packed_ok, wide, wide.cap_qkv_wo, share(tiles_of((int)ro.ptr.size())), &out.dt_wo[l]);
        }
        const l3m_tensor *wu = l3m_file_blk(f, l, "w_up"), *wg = l3m_file_blk(f, l, "w_gate");
        const int ffn_hi = std::min(sr.f_hi * T, (int)wu->shape[0]);
        if (!wg) {                                                                  // GELU MLP: up only
            Rows ru;
            add_rows(ru, f, wu, sr.f_lo * T, ffn_hi, ref);
            out.off_up[l] = pack_rows(s, ru, f, b + "up", out, !packed_ok, wide, wide.cap_rest, share(ftiles), &out.dt_up[l]);
            out.off_gate[l] = (size_t)-1;
            out.dt_gate[l] = out.dt_up[l];
        } else if (ref || wu->dtype == wg->dtype) {
            // Up and gate in one matrix, each CTA's range back to back: [its up tiles][its gate tiles].
            Rows ru;
            for (int c = 0; c < l3m::kClusterCtas; c++) {
                int t0, t1;
                split(ftiles, l3m::kClusterCtas, c, &t0, &t1);
                for (const l3m_tensor *t : {wu, wg}) add_rows(ru, f, t, (sr.f_lo + t0) * T, (sr.f_lo + t1) * T, ref);
            }
            out.off_up[l] = pack_rows(s, ru, f, b + "upgate16", out, !packed_ok, wide, wide.cap_rest, 2 * share(ftiles), &out.dt_up[l]);
            out.off_gate[l] = (size_t)-1;
            out.dt_gate[l] = out.dt_up[l];
        } else {
            Rows ru, rg;
            add_rows(ru, f, wu, sr.f_lo * T, ffn_hi, ref);
            add_rows(rg, f, wg, sr.f_lo * T, ffn_hi, ref);
            out.off_up[l] = pack_rows(s, ru, f, b + "up", out, !packed_ok, wide, wide.cap_rest, share(ftiles), &out.dt_up[l]);
            out.off_gate[l] = pack_rows(s, rg, f, b + "gate", out, !packed_ok, Widen{}, 0, 0, &out.dt_gate[l]);   // read from global memory
        }
        Rows rd;
        const l3m_tensor *wd = l3m_file_blk(f, l, "w_down");
        add_rows(rd, f, wd, sr.d_lo * T, std::min(sr.d_hi * T, (int)wd->shape[0]), ref);
        out.off_down[l] = pack_rows(s, rd, f, b + "down", out, !packed_ok, wide, wide.cap_rest, share(tiles_of((int)rd.ptr.size())), &out.dt_down[l]);
    }
    const l3m_tensor *head = l3m_file_tensor(f, (f->h->flags & L3M_F_TIED) ? "embed" : "lm_head");
    Rows rh;
    add_rows(rh, f, head, sr.v_lo * T, std::min(sr.v_hi * T, (int)head->shape[0]), ref);
    out.off_head = pack_rows(s, rh, f, "head", out, !packed_ok, wide, wide.cap_head, (tiles_of((int)rh.ptr.size()) + wide.head_ctas - 1) / wide.head_ctas, &out.dt_head);
}

// The decode kernel's shared-memory layout for these sizes: every vector's offset in a, the scratch, the
// start of the weight staging area (sm_w) with the attention buffers at its start (w_extra bytes).
// Returns the bytes in use before the staging area's weights; the area itself is the rest of the SM's
// budget. max_tiles, pairs: the largest per-CTA share of a phase (tiles; scratch pairs).
struct LayoutSizes { int dim, ffn, hd, ctx, L, n_qkv, vstride, max_tiles, pairs; bool ln; };
int smem_layout(l3m::DecodeArgs &a, const LayoutSizes &z) {
    const int dim = z.dim, ffn = z.ffn, hd = z.hd, mx = std::max(dim, ffn), nb = (mx + 31) / 32, G = l3m::kClusterCtas;
    int off = 0;
    auto take = [&](int bytes) { int o2 = off; off = align16(off + bytes); return o2; };
    // First what a helper CTA (the head alone) uses, so that its resident head tiles can start at
    // sm_w_head: x, the norm's output and prepared activation, outputs, reductions, the final norm's
    // weights, the layer table (every CTA copies it at entry), the staging barrier, the scratch.
    a.sm_x = take(dim * 4);
    a.sm_xb = take(mx * 4);
    a.sm_tmp = take(mx * 4);
    a.sm_q8 = take(mx);
    a.sm_scale = take(nb * 4);
    a.sm_sum = take(nb * 4);
    a.sm_xf = take(mx * 4);
    a.sm_y = take(z.max_tiles * L3M_TILE * 4);
    a.sm_red = take(64 * 4);
    a.sm_wh = take(dim * 4);
    a.sm_whb = take(z.ln ? dim * 4 : 0);
    a.sm_layers = take(z.L * (int)sizeof(l3m::LayerDev));
    a.sm_wbar = take(16);
    // Scratch: the (scale product, dot) pairs of the largest per-CTA phase of a layer, so each runs in
    // one pass (the head runs in several).
    a.scratch_pairs = z.pairs;
    a.sm_scratch = take(z.pairs * 8);
    off = (off + 127) & ~127;
    a.sm_w_head = off;
    // Then what only the layer cluster uses.
    a.sm_pa_q8 = take(dim);                                            // the q8 exchanges' receive buffers
    a.sm_pa_scale = take((dim / 32 + 1) * 4);
    a.sm_pa_sum = take((dim / 32 + 1) * 4);
    a.sm_ph_q8 = take(ffn);
    a.sm_ph_scale = take((ffn / 32 + 1) * 4);
    a.sm_ph_sum = take((ffn / 32 + 1) * 4);
    a.sm_scores = take(z.ctx * 4);
    a.sm_kv = take(2 * hd * 2);
    a.sm_att = take(hd * 4);
    a.sm_wa = take(dim * 4);
    a.sm_wf = take(dim * 4);
    a.sm_wab = take(z.ln ? dim * 4 : 0);
    a.sm_wfb = take(z.ln ? dim * 4 : 0);
    a.sm_rope = take(hd / 2 * 8);
    a.attn_chunk = std::min(z.ctx, 256);
    a.vstride = z.vstride;
    a.sm_xq = take(z.n_qkv * 4);
    a.sm_xa = take(dim * 4);
    a.sm_xp = take(dim * 4);
    a.sm_xh = take(ffn * 4);
    a.sm_xd = take(dim * 4);
    a.sm_xt = take((4 + 16 * G) * 4);                                  // token, argmax slots, 3 sampling exchanges
    a.sm_xbar = take(5 * 8);
    // The weight staging area takes the rest; the attention buffers are its first bytes.
    off = (off + 127) & ~127;
    a.sm_w = off;
    a.sm_kvbuf = take(a.attn_chunk * (hd + 8) * 2);
    a.sm_vt = take(hd * l3m::attn_vt_stride(a.attn_chunk) * 2);
    off = (off + 127) & ~127;
    a.w_extra = off - a.sm_w;
    return off;
}

// Build everything one GPU holds and fill its decode arguments.
bool build_gpu(l3m_model *m, Gpu &g, const l3m_opts &o) {
    const l3m_file *f = &m->f;
    const bool ref = m->reference;
    if (!cuda_ok(cudaSetDevice(g.dev), "cudaSetDevice")) return false;
    cudaDeviceProp prop;
    if (!cuda_ok(cudaGetDeviceProperties(&prop, g.dev), "cudaGetDeviceProperties")) return false;
    g.name = prop.name;
    g.sms = prop.multiProcessorCount;
    g.l2_bytes = (size_t)prop.l2CacheSize;
    g.persist_max = (size_t)prop.persistingL2CacheMaxSize;
    g.window_max = (size_t)prop.accessPolicyMaxWindowSize;
    if (prop.major != 10) {
        char msg[160];
        snprintf(msg, sizeof msg, "GPU %d (%s) is compute capability %d.%d; this build runs on B200 (sm_100a)", g.dev, prop.name, prop.major, prop.minor);
        fprintf(stderr, "l3m: %s\n", msg);
        return false;
    }
    // One cluster of kClusterCtas CTAs runs the layers; the head runs on every CTA of as many whole
    // clusters as there are SMs for (9 x 16 = 144 on a B200).
    const int G = l3m::kClusterCtas, dim = m->dim, hd = m->hd, ffn = m->ffn, V = m->vocab, L = m->n_layers;
    if (g.sms < G) { fprintf(stderr, "l3m: GPU %d has %d SMs; the decode cluster needs %d\n", g.dev, g.sms, G); return false; }
    int GT = g.sms / G * G;
    // L3M_CLUSTERS=n caps the launch at n clusters (1: the head runs on cluster 0 alone, with no
    // cross-cluster waits; for profilers that do not keep every cluster of a launch resident).
    if (const char *nc = getenv("L3M_CLUSTERS")) GT = std::max(G, std::min(GT, atoi(nc) * G));
    if (hd > l3m::kDecodeThreads) { fprintf(stderr, "l3m: head_dim %d above %d is not built\n", hd, l3m::kDecodeThreads); return false; }
    if (V >= (1 << 24)) { fprintf(stderr, "l3m: a vocabulary of %d entries is not built (the head exchange holds indices below 2^24)\n", V); return false; }

    // Streamed weights first (one contiguous range for the persisting window), then the rest.
    Stage s;
    std::vector<l3m::LayerDev> layers(L);
    Streamed sw;
    const ShardRange sr = shard_range(f->h, m->n_gpus, g.rank);
    const int n_qkv = (m->n_heads + 2 * m->n_kv) * hd;
    const int heads_g = sr.head_hi - sr.head_lo, kv_g = sr.kv_hi - sr.kv_lo, n_qkv_g = (heads_g + 2 * kv_g) * hd;
    Widen wd;                                                            // the staging capacities, from the layout alone
    if (!ref) {
        const int Tq = tiles_of(n_qkv_g), Td = sr.d_hi - sr.d_lo, Tf = sr.f_hi - sr.f_lo, Tv = sr.v_hi - sr.v_lo, mx = std::max(dim, ffn);
        auto share = [&](int t) { return (t + G - 1) / G; };              // the largest of the split's parts
        const int max_t = std::max({tiles_of(3 * hd), share(Tq), 2 * share(Tf), share(Td), share(Tv)});
        const int pr = std::max({(mx / 32) * L3M_TILE, share(Tq) * L3M_TILE * (dim / 32), share(Td) * L3M_TILE * (dim / 32),
                                 2 * share(Tf) * L3M_TILE * (dim / 32), share(Td) * L3M_TILE * (ffn / 32)});
        l3m::DecodeArgs probe{};
        smem_layout(probe, LayoutSizes{dim, ffn, hd, m->ctx, L, n_qkv, (m->ctx + 7) & ~7, max_t, pr, (m->flags & L3M_F_LAYERNORM) != 0});
        const long w_bytes = ((long)l3m_decode_smem_budget() - probe.sm_w) & ~127L;
        wd.on = !getenv("L3M_NO_WIDEN");
        wd.cap_qkv_wo = std::max(0L, w_bytes - probe.w_extra);
        wd.cap_rest = std::max(0L, w_bytes);
        wd.cap_head = std::max(0L, ((long)l3m_decode_smem_budget() - probe.sm_w_head) & ~127L);
        wd.head_ctas = GT > G && !m->cold ? GT - G : GT;
    }
    pack_streamed(f, ref, sr, hd, s, sw, wd);
    const std::vector<size_t> &off_qkv = sw.off_qkv, &off_wo = sw.off_wo, &off_gate = sw.off_gate, &off_up = sw.off_up, &off_down = sw.off_down;
    for (int l = 0; l < L; l++) {
        layers[l].dt_qkv = sw.dt_qkv[l]; layers[l].dt_wo = sw.dt_wo[l]; layers[l].dt_up = sw.dt_up[l];
        layers[l].dt_gate = sw.dt_gate[l]; layers[l].dt_down = sw.dt_down[l];
    }
    const int dt_head = sw.dt_head;
    const size_t off_head = sw.off_head;
    g.weight_bytes = s.buf.size() - sw.widened;                         // the model's bytes, as the reference counts them
    g.held_bytes = s.buf.size();                                         // what the arena holds (widened matrices included)
    const l3m_tensor *emb = l3m_file_tensor(f, "embed");
    int dt_embed = (int)emb->dtype;
    size_t emb_row = l3m_row_bytes(dt_embed, dim), off_embed;
    if (ref && dt_embed != L3M_F32) {
        std::vector<float> rowf((size_t)dim);
        off_embed = s.reserve((size_t)V * dim * 4);
        for (int r = 0; r < V; r++) {
            l3m_dequant_row(rowf.data(), dt_embed, row_ptr(f, emb, r), dim);
            memcpy(s.buf.data() + off_embed + (size_t)r * dim * 4, rowf.data(), (size_t)dim * 4);
        }
        dt_embed = L3M_F32;
        emb_row = (size_t)dim * 4;
    } else {
        off_embed = s.put(l3m_file_data(f, emb), (size_t)V * emb_row);
    }
    auto put_vec = [&](const l3m_tensor *t) -> long long {
        return t ? (long long)s.put(l3m_file_data(f, t), (size_t)t->nbytes) : -1;
    };
    struct VecOffs { long long an, fn, bq, bk, bv, bo, bu, bd, anb, fnb; };
    std::vector<VecOffs> vo(L);
    for (int l = 0; l < L; l++) {
        vo[l] = {put_vec(l3m_file_blk(f, l, "attn_norm")), put_vec(l3m_file_blk(f, l, "ffn_norm")), put_vec(l3m_file_blk(f, l, "bq")),
                 put_vec(l3m_file_blk(f, l, "bk")), put_vec(l3m_file_blk(f, l, "bv")), put_vec(l3m_file_blk(f, l, "bo")),
                 put_vec(l3m_file_blk(f, l, "b_up")), put_vec(l3m_file_blk(f, l, "b_down")), put_vec(l3m_file_blk(f, l, "attn_norm_b")),
                 put_vec(l3m_file_blk(f, l, "ffn_norm_b"))};
    }
    long long off_norm = put_vec(l3m_file_tensor(f, "norm")), off_norm_b = put_vec(l3m_file_tensor(f, "norm_b"));
    long long off_pos = put_vec(l3m_file_tensor(f, "pos_embed"));           // f32 [ctx][dim] (GPT-2 family)
    g.arena_bytes = s.buf.size();

    if (!cuda_ok(cudaMalloc(&g.arena, g.arena_bytes), "weights")) return false;
    if (!cuda_ok(cudaMemcpy(g.arena, s.buf.data(), g.arena_bytes, cudaMemcpyHostToDevice), "weights upload")) return false;
    std::vector<uint8_t>().swap(s.buf);

    // Per layer: K [n_kv][ctx][hd] (a row per position) and V transposed, [n_kv][hd][vstride] (a
    // column per position), both bf16.
    const int vstride = (m->ctx + 7) & ~7;
    const size_t k_per = (size_t)kv_g * m->ctx * hd, v_per = (size_t)kv_g * hd * vstride;   // this GPU's kv heads
    g.kv_bytes = (size_t)L * (k_per + v_per) * 2;
    if (!cuda_ok(cudaMalloc(&g.kv, std::max(g.kv_bytes, (size_t)256)), "KV cache")) return false;
    cudaMemset(g.kv, 0, g.kv_bytes);
    auto A = [&](long long off) -> const float * { return off < 0 ? nullptr : (const float *)(g.arena + off); };
    for (int l = 0; l < L; l++) {
        l3m::LayerDev &d = layers[l];
        d.qkv = g.arena + off_qkv[l];
        d.wo = g.arena + off_wo[l];
        d.up = g.arena + off_up[l];
        d.gate = off_gate[l] == (size_t)-1 ? nullptr : g.arena + off_gate[l];
        d.down = g.arena + off_down[l];
        d.attn_norm = A(vo[l].an); d.ffn_norm = A(vo[l].fn);
        d.attn_norm_b = A(vo[l].anb); d.ffn_norm_b = A(vo[l].fnb);
        d.bq = A(vo[l].bq); d.bk = A(vo[l].bk); d.bv = A(vo[l].bv); d.bo = A(vo[l].bo); d.b_up = A(vo[l].bu); d.b_down = A(vo[l].bd);
        d.kc = g.kv + (size_t)l * (k_per + v_per);
        d.vc = d.kc + k_per;
    }

    auto rope = rope_table(m->ctx, hd, m->f.h->rope_theta);
    if (!cuda_ok(cudaMalloc(&g.rope, rope.size() * sizeof(float2)), "rope")) return false;
    cudaMemcpy(g.rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice);

    // Each CTA's share of every phase: contiguous tile ranges, the reference's split (engine.c:471-476);
    // query heads round-robin over the CTAs.
    const int Td = sr.d_hi - sr.d_lo, Tf = sr.f_hi - sr.f_lo, Tv = sr.v_hi - sr.v_lo, Tq = tiles_of(n_qkv_g);   // this GPU's tiles
    // Roles for a grid of gt CTAs; the shared-memory layout is sized for the largest share (gt = G).
    // helpers_only: the head's tiles go to the helper clusters alone (they keep as many as fit resident
    // in shared memory), else to every CTA.
    auto make_roles = [&](int gt, bool helpers_only = false) {
        std::vector<l3m::Role> rs(gt);
        for (int c = 0; c < gt; c++) {
            l3m::Role &r = rs[c];
            r = l3m::Role{-1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
            if (c < G) {
                r.head0 = c < heads_g ? sr.head_lo + c : -1;
                split(Tq, G, c, &r.qkv0, &r.qkv1);
                split(Td, G, c, &r.wo0, &r.wo1);
                split(Tf, G, c, &r.ffn0, &r.ffn1);
                split(Td, G, c, &r.dn0, &r.dn1);
            }
            if (!helpers_only) split(Tv, gt, c, &r.voc0, &r.voc1);
            else if (c >= G) split(Tv, gt - G, c - G, &r.voc0, &r.voc1);
        }
        return rs;
    };
    int max_tiles = tiles_of(3 * hd);
    for (const l3m::Role &r : make_roles(G))
        max_tiles = std::max({max_tiles, r.qkv1 - r.qkv0, 2 * (r.ffn1 - r.ffn0), r.wo1 - r.wo0, r.dn1 - r.dn0, r.voc1 - r.voc0});

    l3m::DecodeArgs &a = g.args;
    a.dim = dim; a.hd = hd; a.ffn = ffn; a.vocab = V; a.ctx = m->ctx; a.n_heads = m->n_heads; a.n_kv = m->n_kv; a.hpk = m->hpk;
    a.n_layers = L; a.n_qkv = n_qkv; a.grid = GT; a.eps = m->f.h->norm_eps;
    {
        l3m::Shard &h = a.sh;
        h = l3m::Shard{};
        h.n_gpus = m->n_gpus;
        h.gpu = g.rank;
        h.head_lo = sr.head_lo; h.n_heads_g = heads_g; h.kv_lo = sr.kv_lo; h.n_kv_g = kv_g; h.n_qkv_g = n_qkv_g;
        h.d_off = sr.d_lo; h.f_off = sr.f_lo; h.v_off = sr.v_lo;
        for (int r = 0; r < m->n_gpus; r++) {                             // every GPU's slice of each exchanged vector
            const ShardRange o2 = shard_range(f->h, m->n_gpus, r);
            h.lo[l3m::kXAttn][r] = o2.head_lo * hd;
            h.len[l3m::kXAttn][r] = (o2.head_hi - o2.head_lo) * hd;
            h.lo[l3m::kXProj][r] = h.lo[l3m::kXDown][r] = o2.d_lo * L3M_TILE;
            h.len[l3m::kXProj][r] = h.len[l3m::kXDown][r] = std::min(o2.d_hi * L3M_TILE, dim) - o2.d_lo * L3M_TILE;
            h.lo[l3m::kXH][r] = o2.f_lo * L3M_TILE;
            h.len[l3m::kXH][r] = std::min(o2.f_hi * L3M_TILE, ffn) - o2.f_lo * L3M_TILE;
        }
    }
    a.head = g.arena + off_head; a.dt_head = dt_head;
    a.embed = g.arena + off_embed; a.dt_embed = dt_embed; a.embed_row_bytes = (long long)emb_row;
    a.norm = A(off_norm);
    a.norm_b = A(off_norm_b);
    a.cold = m->cold ? 1 : 0;
    a.layernorm = (m->flags & L3M_F_LAYERNORM) ? 1 : 0;
    a.gelu = (m->flags & L3M_F_GELU) ? 1 : 0;
    a.pos_embed = (m->flags & L3M_F_LEARNED_POS) ? A(off_pos) : nullptr;
    a.rope = (m->flags & L3M_F_LEARNED_POS) ? nullptr : g.rope;
    if (l3m_expf_table(&a.etab)) { fprintf(stderr, "l3m: %s\n", l3m_cuda_error()); return false; }
    a.trace_cta[0] = a.trace_cta[1] = -1;
    if (getenv("L3M_TRACE")) {                                         // phase time stamps of two CTAs: a layer CTA and a helper
        const char *tc = getenv("L3M_TRACE_CTA");                      // which layer CTA (default the first)
        a.trace_cta[0] = tc ? atoi(tc) : 0;
        if (a.trace_cta[0] < 0 || a.trace_cta[0] >= l3m::kClusterCtas) {
            fprintf(stderr, "l3m: L3M_TRACE_CTA must be a CTA of the layer cluster, 0..%d\n", l3m::kClusterCtas - 1);
            return false;
        }
        a.trace_cta[1] = GT > G ? G : G - 1;                            // a helper's head, when there are helpers
        g.trace_bytes = (size_t)2 * m->ctx * (L + 1) * l3m::kTraceEvents * sizeof(unsigned long long);
        if (!cuda_ok(cudaMalloc(&g.trace, g.trace_bytes), "trace")) return false;
        cudaMemset(g.trace, 0, g.trace_bytes);
        a.trace = g.trace;
    }
    if (!cuda_ok(cudaMalloc(&g.prompt, (size_t)m->ctx * 4), "prompt")) return false;
    if (!cuda_ok(cudaMalloc(&g.logits, (size_t)m->ctx * V * 4), "logits")) return false;
    if (!cuda_ok(cudaMalloc(&g.probs, (size_t)V * 4), "sampling weights")) return false;
    cudaMemset(g.logits, 0, (size_t)m->ctx * V * 4);
    a.prompt = g.prompt;
    a.eos = m->f.tok.eos; a.bos = m->f.tok.bos;
    a.logits = g.logits;
    // The head exchange (allocated once the grid is known): x (+ the position), the flag, the arrival
    // count, the slots, the abort word.
    const char *tmo = getenv("L3M_TIMEOUT_MS");
    a.hx.timeout_ns = (unsigned long long)(tmo ? atof(tmo) : 5000.0) * 1000000ull;

    // Shared memory layout.
    const int mx = std::max(dim, ffn);
    const bool ln = (m->flags & L3M_F_LAYERNORM) != 0;                   // LayerNorm biases: GPT-2 family only
    int pairs = (mx / 32) * L3M_TILE;
    for (const l3m::Role &r : make_roles(G))
        pairs = std::max({pairs, (r.qkv1 - r.qkv0) * L3M_TILE * (dim / 32), (r.wo1 - r.wo0) * L3M_TILE * (dim / 32),
                          2 * (r.ffn1 - r.ffn0) * L3M_TILE * (dim / 32), (r.dn1 - r.dn0) * L3M_TILE * (ffn / 32)});
    const int off = smem_layout(a, LayoutSizes{dim, ffn, hd, m->ctx, L, n_qkv, vstride, max_tiles, pairs, ln});
    const int budget = l3m_decode_smem_budget();
    if (off > budget) {
        fprintf(stderr, "l3m: dim %d / ffn %d / ctx %d need more shared memory than a B200 SM has for this kernel\n", dim, ffn, m->ctx);
        return false;
    }
    a.w_bytes = (budget - a.sm_w) & ~127;
    a.smem_bytes = a.sm_w + a.w_bytes;
    // How many tiles of each matrix fit in its part of the staging area (qkv and wo: the part past the
    // attention buffers).
    auto fit = [&](int dt, int k, int bytes) { return bytes / (int)l3m::staged_stride(dt, k); };
    for (l3m::LayerDev &d : layers) {
        d.st_qkv = fit(d.dt_qkv, dim, a.w_bytes - a.w_extra);
        d.st_wo = fit(d.dt_wo, dim, a.w_bytes - a.w_extra);
        d.st_up = fit(d.dt_up, dim, a.w_bytes);
        d.st_down = fit(d.dt_down, ffn, a.w_bytes);
    }
    a.st_head = fit(dt_head, dim, (budget - a.sm_w_head) & ~127);     // a helper's: from sm_w_head on
    if (!cuda_ok(cudaMalloc(&g.layers, sizeof(l3m::LayerDev) * L), "layers")) return false;
    cudaMemcpy(g.layers, layers.data(), sizeof(l3m::LayerDev) * L, cudaMemcpyHostToDevice);
    a.layers = g.layers;
    if (o.verbose)
        fprintf(stderr, "l3m: shared memory %d B per CTA: vectors %d, scratch %d pairs, staging %d (attention buffers %d)\n", a.smem_bytes,
                a.sm_scratch, a.scratch_pairs, a.w_bytes, a.w_extra);
    GT = std::min(GT, l3m_decode_occupancy(a.smem_bytes) * G);            // whole clusters resident at once
    if (GT < G) {
        fprintf(stderr, "l3m: a cluster of %d decode CTAs does not fit on GPU %d\n", G, g.dev);
        return false;
    }
    a.grid = GT;
    // The helper clusters keep their head tiles in shared memory (decode.cu head_helper), so unless the
    // weights are read cold, cluster 0 takes none and goes straight from the last layer to the token
    // vote (its own tiles would come from L2 and finish last).
    const bool helpers_only = GT > G && !m->cold;
    a.async_x = !getenv("L3M_CLUSTER_BARRIERS");                        // every CTA of cluster 0 must produce qkv rows
    {
        std::vector<l3m::Role> rs0 = make_roles(GT, helpers_only);
        for (int c = 0; c < G; c++)
            if (rs0[c].qkv0 >= rs0[c].qkv1) a.async_x = 0;
        // Prepared exchanges (one GPU, st.async exchanges; L3M_FLOAT_EXCHANGES=1 keeps plain floats). The
        // q8 form needs whole blocks from every producer: a head's hd outputs, each ffn CTA's rows; and
        // quantised wo / down in every layer (the activation is then the q8 prepare's).
        const bool prepared = a.async_x && m->n_gpus == 1 && !getenv("L3M_FLOAT_EXCHANGES");
        bool wo_q = true, down_q = true;
        for (const l3m::LayerDev &d : layers) {
            wo_q = wo_q && d.dt_wo >= l3m::DT_Q8;
            down_q = down_q && d.dt_down >= l3m::DT_Q8;
        }
        bool ffn_blocks = ffn % 32 == 0;
        for (int c = 0; c < G; c++) {
            const l3m::Role &r = rs0[c];
            if (r.ffn0 >= r.ffn1) continue;
            const int g0 = r.ffn0 * L3M_TILE, n = std::min(r.ffn1 * L3M_TILE, ffn) - g0;
            if (g0 % 32 || n % 32) ffn_blocks = false;
        }
        // Float matrices: the producers round to the matrix's prepare form, when every layer's matrix is
        // that same float dtype.
        auto float_form = [&](bool is_wo) {
            const int d0 = is_wo ? layers[0].dt_wo : layers[0].dt_down;
            if (d0 != l3m::DT_F32 && d0 != l3m::DT_BF16) return (int)l3m::kXFloat;
            for (const l3m::LayerDev &d : layers)
                if ((is_wo ? d.dt_wo : d.dt_down) != d0) return (int)l3m::kXFloat;
            return d0 == l3m::DT_BF16 ? (int)l3m::kXPrepBF16 : (int)l3m::kXPrepF32;
        };
        a.qx_attn = !prepared ? l3m::kXFloat : wo_q && hd % 32 == 0 && dim % 32 == 0 ? l3m::kXQ8 : float_form(true);
        a.qx_h = !prepared ? l3m::kXFloat : down_q && ffn_blocks ? l3m::kXQ8 : float_form(false);
    }
    {
        std::vector<l3m::Role> roles = make_roles(GT, helpers_only);
        if (!cuda_ok(cudaMalloc(&g.roles, sizeof(l3m::Role) * GT), "roles")) return false;
        cudaMemcpy(g.roles, roles.data(), sizeof(l3m::Role) * GT, cudaMemcpyHostToDevice);
        a.roles = g.roles;
    }
    {                                                                  // x words, abort word, slots, statistics
        const size_t x_bytes = ((size_t)(dim + 1) * 8 + 255) & ~(size_t)255, slot_bytes = ((size_t)GT * 8 + 255) & ~(size_t)255;
        g.hx_bytes = x_bytes + 256 + slot_bytes + l3m::kClusterCtas * 8;
        if (!cuda_ok(cudaMalloc(&g.hx, g.hx_bytes), "head exchange")) return false;
        char *b = (char *)g.hx;
        a.hx.xw = (unsigned long long *)b;
        a.hx.abort_flag = (int *)(b + x_bytes);
        a.hx.slots = (unsigned long long *)(b + x_bytes + 256);
        a.hx.stats = (unsigned long long *)(b + x_bytes + 256 + slot_bytes);
    }
    a.slot_lo = helpers_only ? G : 0;
    if (m->cold) {                                                     // 1.5 x L2, in whole copies per CTA of the cluster
        a.cold_chunk = std::min(a.w_extra, 64 << 10) & ~15;
        const unsigned long long unit = (unsigned long long)G * a.cold_chunk;
        a.cold_bytes = (g.l2_bytes * 3 / 2 + unit - 1) / unit * unit;
        if (a.cold_chunk < 4096 || !cuda_ok(cudaMalloc(&g.cold, a.cold_bytes), "cold-mode scratch")) return false;
        a.cold_buf = g.cold;
    }
    a.ctrl = m->ctrl_dev + g.rank;
    a.tokens = m->tokens_dev;
    if (m->n_gpus > 1) {                                               // what the other GPUs write into (zeroed: epoch 0 never matches)
        g.rx_bytes = (size_t)2 * (3 * dim + ffn) * sizeof(unsigned long long);
        g.vote_bytes = (size_t)2 * l3m::kMaxShardGpus * 2 * sizeof(unsigned long long);
        if (!cuda_ok(cudaMalloc(&g.rx, g.rx_bytes), "exchange buffers") || !cuda_ok(cudaMalloc(&g.vote, g.vote_bytes), "vote buffers"))
            return false;
        cudaMemset(g.rx, 0, g.rx_bytes);
        cudaMemset(g.vote, 0, g.vote_bytes);
    }
    if (!cuda_ok(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking), "stream")) return false;
    if (!cuda_ok(cudaStreamCreateWithFlags(&g.side, cudaStreamNonBlocking), "stream")) return false;
    if (!cuda_ok(cudaMalloc(&g.args_dev, sizeof(l3m::DecodeArgs)), "args")) return false;
    cudaEventCreate(&g.ev0);
    cudaEventCreate(&g.ev1);
    (void)o;
    return true;
}

// Keep the streamed weights in L2 with a persisting access-policy window (the GPU form of the
// reference's cache residency). Returns false when over budget and not forced.
bool place_in_l2(l3m_model *m, Gpu &g, const l3m_opts &o, bool *over) {
    *over = g.weight_bytes > g.persist_max;
    if (o.verbose || (*over && !o.force))
        fprintf(stderr, "l3m: gpu %d (%s)  heads [0, %d)  weights %.2f + kv %.2f MiB, persisting L2 budget %.2f of %.2f MiB L2%s\n",
                g.dev, g.name.c_str(), m->n_heads, g.weight_bytes / MiB, g.kv_bytes / MiB, g.persist_max / MiB, g.l2_bytes / MiB,
                *over ? "  OVER" : "");
    if (*over && !o.force) return false;
    if (m->cold || !g.persist_max || !g.window_max) return true;
    cudaSetDevice(g.dev);
    size_t setaside = std::min(g.held_bytes, g.persist_max);
    // The window is best effort (the decode is correct without it), but a failure to set it is reported.
    cudaError_t e = cudaDeviceGetLimit(&g.prev_limit, cudaLimitPersistingL2CacheSize);
    if (e == cudaSuccess) e = cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, setaside);
    if (e == cudaSuccess) {
        g.limit_set = true;
        cudaStreamAttrValue attr = {};
        attr.accessPolicyWindow.base_ptr = g.arena;
        attr.accessPolicyWindow.num_bytes = std::min(g.held_bytes, g.window_max);
        attr.accessPolicyWindow.hitRatio = (float)std::min(1.0, (double)setaside / attr.accessPolicyWindow.num_bytes);
        attr.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
        attr.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
        e = cudaStreamSetAttribute(g.stream, cudaStreamAttributeAccessPolicyWindow, &attr);
    }
    if (e != cudaSuccess) {
        fprintf(stderr, "l3m: gpu %d: persisting L2 window not set (%s); the weights compete for L2\n", g.dev, cudaGetErrorString(e));
        cudaGetLastError();
    } else if (o.verbose) {
        fprintf(stderr, "l3m: gpu %d: persisting L2 window over %.2f MiB of weights, %.2f MiB set aside\n", g.dev,
                std::min(g.held_bytes, g.window_max) / MiB, setaside / MiB);
    }
    return true;
}

// Several GPUs: peer access both ways between every pair, then every GPU's arguments get every
// GPU's receive buffers, vote buffer, logits history and abort word.
bool connect_gpus(l3m_model *m) {
    for (int i = 0; i < m->n_gpus; i++) {
        cudaSetDevice(m->g[i].dev);
        for (int j = 0; j < m->n_gpus; j++) {
            if (i == j) continue;
            cudaError_t e = cudaDeviceEnablePeerAccess(m->g[j].dev, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (!cuda_ok(e, "peer access")) return false;
        }
    }
    for (int i = 0; i < m->n_gpus; i++) {
        l3m::Shard &h = m->g[i].args.sh;
        for (int j = 0; j < m->n_gpus; j++) {
            const Gpu &o = m->g[j];
            const int dim = m->dim;
            unsigned long long *base = o.rx;                           // [kind][2 halves][length]
            h.rx[j][l3m::kXAttn] = base;
            h.rx[j][l3m::kXProj] = base + 2 * (size_t)dim;
            h.rx[j][l3m::kXDown] = base + 4 * (size_t)dim;
            h.rx[j][l3m::kXH] = base + 6 * (size_t)dim;
            h.vote[j] = o.vote;
            h.logits[j] = o.logits;
            h.abort[j] = o.args.hx.abort_flag;
        }
    }
    return true;
}

// What the decode kernel recorded about the first failure of a launch.
void report_decode_error(const l3m::Ctrl *c) {
    const int e = c->error;
    if (!c->done) {
        fprintf(stderr, "l3m: decode kernel did not finish\n");
    } else if (e == l3m::kErrShape) {
        fprintf(stderr, "l3m: decode kernel launched with %d CTAs per cluster, %d clusters, grid %d, block %d; it needs clusters of %d "
                "CTAs of %d threads (code %d)\n", c->where[0], c->where[1], c->where[2], c->where[3], l3m::kClusterCtas,
                l3m::kDecodeThreads, e);
    } else {
        static const char *waits[] = {"?", "exchange 1 (qkv)", "exchange 2 (attention)", "exchange 3 (wo)", "exchange 4 (ffn gate)",
                                      "exchange 5 (down)", "?", "?", "a weight copy", "the published x", "the posted head slots"};
        const int w = c->where[3];
        const char *what = e == l3m::kErrTimeout ? "a wait on another CTA gave up" : e == l3m::kErrStageTimeout ? "a weight copy wait gave up"
                           : e == l3m::kErrToken ? "a sampled token outside the vocabulary" : "unknown error";
        if (e == l3m::kErrToken)
            fprintf(stderr, "l3m: decode kernel: %s (token %d at position %d, code %d)\n", what, w, c->where[1], e);
        else
            fprintf(stderr, "l3m: decode kernel: %s: CTA %d, position %d, layer %d, waiting for %s (code %d)\n", what, c->where[0],
                    c->where[1], c->where[2], w >= 0 && w <= 10 ? waits[w] : "?", e);
    }
}

}  // namespace

extern "C" {

// Write `out`: the file `in` unchanged, then every streamed matrix packed as the decode kernel reads
// it ("b200v1." tensors, whose bytes equal a row-major matrix of the same shape and dtype, so a v1
// reader accepts and ignores them), then a new table of contents; the header's tensor count and
// table offset are updated. The written file is read back and must pack to the same bytes.
L3M_API int l3m_write_packed(const char *in, const char *out) {
    l3m_file f;
    if (l3m_file_open(&f, in)) return -1;
    const l3m_header *h = f.h;
    const int hd = (int)(h->dim / h->n_heads);
    Stage s;
    Streamed sw;
    pack_streamed(&f, false, shard_range(h, 1, 0), hd, s, sw);
    std::vector<l3m_tensor> toc;
    for (uint32_t i = 0; i < h->n_tensors; i++)
        if (strncmp(f.toc[i].name, kPackedPrefix, strlen(kPackedPrefix))) toc.push_back(f.toc[i]);
    FILE *o = fopen(out, "wb");
    bool ok = o && fwrite(f.map, 1, f.size, o) == f.size;
    size_t pos = f.size;
    auto pad = [&](size_t a) {
        static const uint8_t z[64] = {0};
        const size_t n = (a - pos % a) % a;
        ok = ok && fwrite(z, 1, n, o) == n;
        pos += n;
    };
    for (const Streamed::Entry &e : sw.entries) {
        pad(64);
        l3m_tensor t = {};
        snprintf(t.name, sizeof t.name, "%s%s", kPackedPrefix, e.name.c_str());
        t.dtype = (uint32_t)e.dtype;
        t.ndim = 2;
        t.shape[0] = e.rows;
        t.shape[1] = (uint64_t)e.k;
        t.offset = pos;
        t.nbytes = e.rows / L3M_TILE * l3m_tile_bytes(e.dtype, e.k);
        ok = ok && fwrite(s.buf.data() + e.off, 1, t.nbytes, o) == t.nbytes;
        pos += t.nbytes;
        toc.push_back(t);
    }
    pad(8);
    l3m_header nh = *h;
    nh.n_tensors = (uint32_t)toc.size();
    nh.toc_offset = pos;
    ok = ok && fwrite(toc.data(), sizeof(l3m_tensor), toc.size(), o) == toc.size();
    ok = ok && fseek(o, 0, SEEK_SET) == 0 && fwrite(&nh, sizeof nh, 1, o) == 1;
    if (o) ok = fclose(o) == 0 && ok;
    l3m_file_close(&f);
    if (!ok) { fprintf(stderr, "l3m: %s: write failed\n", out); return -1; }
    l3m_file g;                                                       // read back: the packed tensors must be taken as they are
    if (l3m_file_open(&g, out)) return -1;
    Stage s2;
    Streamed sw2;
    pack_streamed(&g, false, shard_range(g.h, 1, 0), hd, s2, sw2);
    l3m_file_close(&g);
    if (s2.buf != s.buf) { fprintf(stderr, "l3m: %s: the packed section does not read back as written\n", out); return -1; }
    return 0;
}

L3M_API l3m_model *l3m_load(const char *path, const l3m_opts *opts) {
    l3m_opts o = opts ? *opts : l3m_opts{};
    l3m_model *m = new l3m_model();
    if (l3m_file_open(&m->f, path)) { delete m; return nullptr; }
    const l3m_header *h = m->f.h;
    m->flags = h->flags;
    m->dim = (int)h->dim; m->n_heads = (int)h->n_heads; m->n_kv = (int)h->n_kv_heads; m->hpk = m->n_heads / m->n_kv;
    m->hd = m->dim / m->n_heads; m->ffn = (int)h->ffn_dim; m->vocab = (int)h->vocab; m->n_layers = (int)h->n_layers;
    m->ctx = std::min((int)h->ctx, o.ctx > 0 ? o.ctx : kDefaultCtx);
    m->reference = o.reference;
    m->cold = o.cold;
    m->kk = l3m_kernels_pick();
    if (m->kk != &l3m_kernels_sm100a) return fail(m, "the decode engine runs the sm100a (exact) table; unset L3M_ISA");
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices < 1) return fail(m, "no CUDA device: this build runs on B200 GPUs only");
    int list[kMaxGpus], n = o.cpus ? o.n_cpus : 1;
    if (n < 1 || n > kMaxGpus) return fail(m, "bad GPU list");
    for (int i = 0; i < n; i++) {
        list[i] = o.cpus ? o.cpus[i] : 0;
        if (list[i] < 0 || list[i] >= devices) return fail(m, "bad GPU list: no such device");
        for (int j = 0; j < i; j++) if (list[j] == list[i]) return fail(m, "a GPU appears twice in the list");
    }
    if (n > l3m::kMaxShardGpus) return fail(m, "bad GPU list: at most 8 GPUs");
    if (n > 1) {
        // Every GPU must produce a slice of the dim and ffn vectors each layer (the exchange buffers'
        // reuse rests on it), and every pair must reach the other's memory.
        if (tiles_of(m->dim) < n || tiles_of(m->ffn) < n) return fail(m, "dim or ffn has fewer 16-row tiles than GPUs: use fewer GPUs");
        for (int i = 0; i < n; i++)
            for (int j = 0; j < n; j++) {
                int can = 0;
                if (i != j && (cudaDeviceCanAccessPeer(&can, list[i], list[j]) != cudaSuccess || !can))
                    return fail(m, "a GPU of the list cannot access another's memory (no peer access between them)");
            }
    }
    m->n_gpus = n;
    cudaSetDevice(list[0]);
    if (!cuda_ok(cudaHostAlloc((void **)&m->ctrl, sizeof(l3m::Ctrl) * kMaxGpus, cudaHostAllocMapped | cudaHostAllocPortable), "control block") ||
        !cuda_ok(cudaHostAlloc((void **)&m->tokens, (size_t)m->ctx * 4, cudaHostAllocMapped | cudaHostAllocPortable), "token ring"))
        return fail(m, "host-mapped memory unavailable");
    cudaHostGetDevicePointer((void **)&m->ctrl_dev, m->ctrl, 0);
    cudaHostGetDevicePointer((void **)&m->tokens_dev, m->tokens, 0);
    bool over_any = false;
    for (int i = 0; i < n; i++) {
        m->g[i].dev = list[i];
        m->g[i].rank = i;
        if (!build_gpu(m, m->g[i], o)) { l3m_free(m); return nullptr; }
        bool over;
        if (!place_in_l2(m, m->g[i], o, &over)) {
            over_any = true;
        }
        m->weight_bytes += m->g[i].weight_bytes;
    }
    if (n > 1 && !connect_gpus(m)) { l3m_free(m); return nullptr; }
    if (over_any) {
        char msg[256];
        snprintf(msg, sizeof msg, "the weights will not stay resident in the persisting L2 window on %d GPU%s: use more GPUs, "
                 "a smaller --dtype at export, or --force", n, n > 1 ? "s" : "");
        return fail(m, msg);
    }
    m->host_logits.assign((size_t)m->vocab, 0.0f);
    const char *base = strrchr(path, '/');
    base = base ? base + 1 : path;
    const int dtype = (int)l3m_file_blk(&m->f, 0, "w_up")->dtype;
    if (m->reference)
        snprintf(m->desc, sizeof m->desc, "%s: %s, %d layers, reference fp32 on %d GPU%s (%s)", base, l3m_dtype_name(dtype), m->n_layers, n,
                 n > 1 ? "s" : "", m->kk->name);
    else
        snprintf(m->desc, sizeof m->desc, "%s: %s, %d layers, %.1f MiB on %d GPU%s (%s)", base, l3m_dtype_name(dtype), m->n_layers,
                 m->weight_bytes / MiB, n, n > 1 ? "s" : "", m->kk->name);
    if (o.verbose) fprintf(stderr, "l3m: %s, ctx %d\n", m->desc, m->ctx);
    return m;
}

L3M_API void l3m_free(l3m_model *m) {
    if (!m) return;
    for (int i = 0; i < kMaxGpus; i++) {
        Gpu &g = m->g[i];
        if (g.dev < 0) continue;
        cudaSetDevice(g.dev);
        if (g.stream) cudaStreamSynchronize(g.stream);
        if (g.limit_set) {
            cudaCtxResetPersistingL2Cache();
            cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, g.prev_limit);
        }
        cudaFree(g.arena); cudaFree(g.kv); cudaFree(g.rope); cudaFree(g.layers); cudaFree(g.roles); cudaFree(g.args_dev); cudaFree(g.trace); cudaFree(g.hx); cudaFree(g.cold);
        cudaFree(g.prompt); cudaFree(g.logits); cudaFree(g.probs); cudaFree(g.rx); cudaFree(g.vote);
        if (g.ev0) cudaEventDestroy(g.ev0);
        if (g.ev1) cudaEventDestroy(g.ev1);
        if (g.stream) cudaStreamDestroy(g.stream);
        if (g.side) cudaStreamDestroy(g.side);
    }
    if (m->ctrl) cudaFreeHost(m->ctrl);
    if (m->tokens) cudaFreeHost(m->tokens);
    l3m_file_close(&m->f);
    delete m;
}

L3M_API int l3m_generate(l3m_model *m, const int32_t *prompt, int n_prompt, int max_new, float temperature, uint64_t seed,
                         int (*on_token)(int32_t, void *), void *user) {
    if (n_prompt < 1 || n_prompt >= m->ctx) return 0;
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= m->vocab) { fprintf(stderr, "l3m: token %d out of range\n", prompt[i]); return -1; }
    Gpu &g = m->g[0];
    memset((void *)m->ctrl, 0, sizeof(l3m::Ctrl) * kMaxGpus);
    // Exchange epochs: every layer step and sampled position of this launch gets epochs no earlier
    // launch used; before they would wrap, the (idle) exchange buffers are cleared and they restart.
    const uint32_t span = (uint32_t)m->ctx * (uint32_t)(m->n_layers + 1) + 64;
    if (m->n_gpus > 1 && m->epoch_next > 0x3F000000u - span) {
        for (int i = 0; i < m->n_gpus; i++) {
            cudaSetDevice(m->g[i].dev);
            cudaMemset(m->g[i].rx, 0, m->g[i].rx_bytes);
            cudaMemset(m->g[i].vote, 0, m->g[i].vote_bytes);
            cudaDeviceSynchronize();
        }
        m->epoch_next = 1;
    }
    const uint32_t epoch0 = m->epoch_next;
    m->epoch_next += span;
    const double t0 = now_ns();
    for (int i = m->n_gpus - 1; i >= 0; i--) {                          // GPU 0 last: its events time the call
        Gpu &gi = m->g[i];
        cudaSetDevice(gi.dev);
        l3m::DecodeArgs a = gi.args;
        a.n_prompt = n_prompt;
        a.max_new = max_new;
        a.temp = temperature > 0 ? temperature : 0.0f;                 // NaN and <= 0: greedy (reference engine.c:301)
        a.rng = seed * 0x9E3779B97F4A7C15ULL + 1;                       // reference engine.c:555
        a.probs = gi.probs;
        a.sh.epoch0 = epoch0;
        a.sh.all_logits = a.temp > 0.0f;                               // every GPU samples from the whole row
        cudaMemcpyAsync(gi.prompt, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, gi.stream);
        cudaMemcpyAsync(gi.args_dev, &a, sizeof a, cudaMemcpyHostToDevice, gi.stream);
        cudaMemsetAsync(gi.hx, 0, gi.hx_bytes, gi.stream);              // no head word carries an epoch; abort word 0
        cudaEventRecord(gi.ev0, gi.stream);
        if (l3m_decode_launch(&a, gi.args_dev, gi.stream)) return -1;
        cudaEventRecord(gi.ev1, gi.stream);
    }
    cudaSetDevice(g.dev);
    int seen = 0, n_gen = 0, stopped = -1;
    if (on_token) {
        for (;;) {
            const int done = m->ctrl->done;
            const int np = m->ctrl->n_published;
            for (; seen < np; seen++) {
                if (stopped >= 0) continue;
                n_gen++;
                m->logits_pos = n_prompt - 1 + seen;                 // l3m_logits inside on_token: this token's logits
                // A volatile read, after the volatile read of n_published: the compiler keeps the
                // order and x86 does not reorder loads, so the token is the one the kernel published.
                const int32_t tok = ((volatile const int32_t *)m->tokens)[seen];
                if (!on_token(tok, user)) {
                    stopped = seen;
                    m->ctrl->stop_request = 1;
                }
            }
            if (done) break;
            // The kernel ended without finishing its loop, or failed (a CUDA error, reported below by
            // the stream synchronisation): stop polling either way.
            const cudaError_t q = cudaEventQuery(g.ev1);
            if (q != cudaErrorNotReady && !m->ctrl->done) break;
            _mm_pause();
        }
    }
    cudaError_t e = cudaStreamSynchronize(g.stream);
    const double t1 = now_ns();
    for (int i = 1; i < m->n_gpus && e == cudaSuccess; i++) {
        cudaSetDevice(m->g[i].dev);
        e = cudaStreamSynchronize(m->g[i].stream);
    }
    cudaSetDevice(g.dev);
    if (!cuda_ok(e, "decode")) return -1;
    for (int i = 0; i < m->n_gpus; i++) {
        const l3m::Ctrl *c = m->ctrl + i;
        if (!c->done || c->error) {
            if (m->n_gpus > 1) fprintf(stderr, "l3m: GPU %d of %d:\n", i, m->n_gpus);
            report_decode_error(c);
            return -1;
        }
    }
    int last_pos;
    if (stopped >= 0) {
        last_pos = n_prompt - 1 + stopped;
    } else {
        n_gen = m->ctrl->n_gen;
        last_pos = m->ctrl->final_pos;
    }
    m->logits_pos = last_pos;
    m->cached_pos = -2;
    if (g.trace) {                                                      // L3M_TRACE: raw stamps for offline analysis
        std::vector<unsigned long long> t(g.trace_bytes / 8);
        cudaMemcpy(t.data(), g.trace, g.trace_bytes, cudaMemcpyDeviceToHost);
        if (FILE *tf = fopen(getenv("L3M_TRACE"), "wb")) {
            int khz = 0;                                                 // the stamps are SM cycles; the header carries the clock
            cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, g.dev);
            int hdr[8] = {m->ctx, m->n_layers, n_prompt, last_pos, g.args.trace_cta[0], g.args.trace_cta[1], l3m::kTraceEvents, khz};
            fwrite(hdr, sizeof hdr, 1, tf);
            fwrite(t.data(), 8, t.size(), tf);
            fclose(tf);
        }
    }
    float ms = 0;
    cudaEventElapsedTime(&ms, g.ev0, g.ev1);
    // GPU 0's launch statistics: the layer cluster's wait cycles (averaged over its CTAs, the reference's
    // average over ranks) at this launch's cycles-to-time ratio, and the cold flushes' time.
    const l3m::Ctrl *c0 = m->ctrl;
    const double cyc = (double)(c0->cyc1 - c0->cyc0), gt = (double)(c0->gt1 - c0->gt0);
    const double ns_per_cyc = cyc > 0 && gt > 0 ? gt / cyc : 0.0;
    m->tok_count += last_pos + 1;
    m->ns += t1 - t0;
    m->dev_ns += ms * 1e6;
    m->wait_ns += (double)c0->wait_cyc / l3m::kClusterCtas * ns_per_cyc;
    m->cold_ns += (double)c0->cold_ns;
    return n_gen;
}

L3M_API const float *l3m_logits(const l3m_model *cm) {
    l3m_model *m = const_cast<l3m_model *>(cm);
    if (m->logits_pos >= 0 && m->cached_pos != m->logits_pos) {
        Gpu &g = m->g[0];
        cudaSetDevice(g.dev);
        cudaMemcpyAsync(m->host_logits.data(), g.logits + (size_t)m->logits_pos * m->vocab, (size_t)m->vocab * 4, cudaMemcpyDeviceToHost, g.side);
        cudaStreamSynchronize(g.side);
        m->cached_pos = m->logits_pos;
    }
    return m->host_logits.data();
}

L3M_API int l3m_vocab(const l3m_model *m) { return m->vocab; }
L3M_API int l3m_ctx(const l3m_model *m) { return m->ctx; }
L3M_API const char *l3m_describe(const l3m_model *m) { return m->desc; }
L3M_API int l3m_bos(const l3m_model *m) { return m->f.tok.bos; }
L3M_API int l3m_eos(const l3m_model *m) { return m->f.tok.eos; }
L3M_API const char *l3m_chatml(const l3m_model *m, int32_t *im_start) {
    *im_start = m->f.im_start;
    return m->f.system;
}
L3M_API int l3m_encode(const l3m_model *m, const char *text, int add_bos, int32_t *out, int max) {
    return l3m_tokenizer_encode(&m->f.tok, text, add_bos, out, max);
}
L3M_API const char *l3m_decode(const l3m_model *m, int32_t tok, int *len) {
    return (const char *)l3m_tokenizer_decode(&m->f.tok, tok, len);
}

// The reference's accounting (src/engine.c:578-593): token time excludes the cold flushes; ns_wait is
// the time the workers (here the layer cluster's CTAs, averaged) spent in exchange and token waits;
// ns_compute is the rest.
L3M_API int l3m_perf_read(l3m_model *m, l3m_perf *out) {
    memset(out, 0, sizeof *out);
    out->l3_miss = out->dram_bytes = out->energy_j = out->llc_occupancy = NAN;
    const double tokens = m->tok_count, ns = std::max(0.0, m->ns - m->cold_ns), wait = m->wait_ns;
    m->tok_count = m->ns = m->dev_ns = m->wait_ns = m->cold_ns = 0;
    if (tokens <= 0) return -1;
    out->tokens = tokens;
    out->ns_token = ns / tokens;
    out->ns_wait = std::min(wait / tokens, out->ns_token);
    out->ns_compute = out->ns_token - out->ns_wait;
    out->bytes_token = (double)m->weight_bytes;
    for (int i = 0; i < m->n_gpus; i++) out->l2_bytes += (double)m->g[i].l2_bytes;
    return 0;
}

L3M_API double l3m_device_ns(const l3m_model *m) { return std::max(0.0, m->dev_ns - m->cold_ns); }

L3M_API int l3m_parse_cpus(const char *list, int *cpus, int max) {
    int n = 0;
    const char *p = list;
    if (!p || !*p) return -1;
    for (;;) {
        char *end;
        long a = strtol(p, &end, 10);
        if (end == p || a < 0 || a > 4095) return -1;
        long b = a;
        p = end;
        if (*p == '-') {
            b = strtol(p + 1, &end, 10);
            if (end == p + 1 || b < a || b > 4095) return -1;
            p = end;
        }
        for (long c = a; c <= b; c++) {
            if (n == max) return -1;
            cpus[n++] = (int)c;
        }
        if (!*p) return n;
        if (*p != ',' || !p[1]) return -1;
        p++;
    }
}

L3M_API void l3m_print_hw(FILE *out) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) { fprintf(out, "no CUDA devices\n"); return; }
    for (int d = 0; d < n; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) != cudaSuccess) continue;
        fprintf(out, "GPU %d: %s, sm_%d%d, %d SMs, L2 %.1f MiB, persisting budget %.1f MiB, window %.1f MiB, %.1f GiB\n", d, p.name,
                p.major, p.minor, p.multiProcessorCount, p.l2CacheSize / MiB, p.persistingL2CacheMaxSize / MiB,
                p.accessPolicyMaxWindowSize / MiB, p.totalGlobalMem / (MiB * 1024));
    }
}

}  // extern "C"
