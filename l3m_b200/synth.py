"""Seeded synthetic .l3m models for the benchmark and parity configurations.

The .l3m container (header, 64-byte aligned tensors, table of contents, tokenizer) and the ggml
block quantisers are the reference's on-disk format (fpedd/l3m src/model.h:3-70; its writer is
python/l3m/export.py:73-100 and its quantisers export.py:175-208). This module writes that format
itself, so the GPU box needs no copy of the reference; tests pin it byte-for-byte against the
reference's own exporter and ggml golden vectors.

Weights follow the recipe of the benchmark configurations: N(0, 0.02) fp32 tensors drawn in a fixed
order from numpy.random.default_rng(seed), norm gains 1.0, a byte-level tokenizer (256 bytes, <s>,
</s>, empty pieces up to vocab), then quantised per 32-element block by the file dtype.
"""
import os
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

DTYPES = {"f32": 0, "bf16": 1, "q8_0": 2, "q4_0": 3, "mxfp4": 4}
LAYERNORM, LEARNED_POS, GELU, TIED, SP_PREFIX, DIGITS = 1, 2, 4, 8, 16, 32
NO_MERGE = -1e9
MXFP4_LUT = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], dtype=np.float32)   # doubled e2m1


# ---- ggml block quantisers (bytes identical to ggml's quantize_row_*_ref)

def to_bf16(x):
    """fp32 -> bf16 bits, round to nearest even; NaN stays NaN."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    rne = (u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16
    return np.where(np.isnan(x), (u >> 16) | 0x40, rne).astype(np.uint16)


def _round_half_away(x):
    return np.sign(x) * np.floor(np.abs(x).astype(np.float64) + 0.5)


def _recip(d):
    """ggml multiplies by 1/d (in fp32), which rounds differently from dividing by d."""
    safe = np.where(d != 0, d, np.float32(1))
    return np.where(d != 0, np.float32(1) / safe, np.float32(0)).astype(np.float32)


def q8_0(x):
    b = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    d = (np.abs(b).max(axis=1) / np.float32(127)).astype(np.float32)
    q = _round_half_away(b * _recip(d)[:, None]).astype(np.int8)
    return np.concatenate([d.astype(np.float16).view(np.uint8).reshape(-1, 2), q.view(np.uint8)], axis=1)


def q4_0(x):
    b = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    signed_max = b[np.arange(len(b)), np.abs(b).argmax(axis=1)]
    d = (signed_max / np.float32(-8)).astype(np.float32)
    q = np.clip(np.floor(b * _recip(d)[:, None] + np.float32(8.5)), 0, 15).astype(np.uint8)
    return np.concatenate([d.astype(np.float16).view(np.uint8).reshape(-1, 2), q[:, :16] | (q[:, 16:] << 4)], axis=1)


def mxfp4(x):
    b = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(b).max(axis=1)
    e = np.where(amax > 0, np.floor(np.log2(np.where(amax > 0, amax, 1))) - 2 + 127, 0).astype(np.uint8)
    d = np.ldexp(0.5, e.astype(np.int32) - 127)                      # 2^(e-127) / 2
    q = np.abs(b[:, :, None] - MXFP4_LUT * d[:, None, None]).argmin(axis=2).astype(np.uint8)
    return np.concatenate([e[:, None], q[:, :16] | (q[:, 16:] << 4)], axis=1)


def encode(x, dtype):
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.tobytes()
    if dtype == "bf16":
        return to_bf16(x).tobytes()
    if x.shape[-1] % 32:
        raise ValueError(f"{dtype}: inputs {x.shape[-1]} not a multiple of 32")
    fn = {"q8_0": q8_0, "q4_0": q4_0, "mxfp4": mxfp4}[dtype]
    flat = x.reshape(-1, 32)
    step = 1 << 18                                        # blocks per chunk: bounded temporaries
    return b"".join(fn(flat[i:i + step]).tobytes() for i in range(0, len(flat), step))


# ---- the container

@dataclass
class Model:
    arch: str
    flags: int
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    ffn_dim: int
    vocab: int
    ctx: int
    rope_theta: float
    norm_eps: float
    tensors: dict = field(default_factory=dict)      # canonical name -> fp32 array
    tokens: list = field(default_factory=list)       # (bytes, score) per id
    bos: int = -1
    eos: int = -1


def tensor_dtype(name, m, dtype, head_dtype):
    """Vectors and pos_embed stay f32; the head (the embedding when tied) takes head_dtype; an
    untied embedding is f32 (it is gathered, not streamed); every other matrix takes dtype."""
    if m.tensors[name].ndim == 1 or name == "pos_embed":
        return "f32"
    if name == "lm_head" or (name == "embed" and m.flags & TIED):
        return head_dtype
    return "f32" if name == "embed" else dtype


def write(m, dtype, head_dtype, out):
    """Write m as a .l3m v1 file. Returns {tensor name: bytes}."""
    names = sorted(m.tensors)
    dts = {n: tensor_dtype(n, m, dtype, head_dtype) for n in names}
    blobs = {n: encode(m.tensors[n], dts[n]) for n in names}
    max_len = max(len(b) for b, _ in m.tokens)
    with open(out, "wb") as f:
        f.write(bytes(1024))
        toc = []
        for n in names:
            f.seek((f.tell() + 63) // 64 * 64)
            t = m.tensors[n]
            shape = list(t.shape) + [0] * (4 - t.ndim)
            toc.append(struct.pack("<64sII4QQQ", n.encode(), DTYPES[dts[n]], t.ndim, *shape, f.tell(), len(blobs[n])))
            f.write(blobs[n])
        f.seek((f.tell() + 7) // 8 * 8)
        toc_offset = f.tell()
        f.write(b"".join(toc))
        tok_offset = f.tell()
        f.write(struct.pack("<IiiI", len(m.tokens), m.bos, m.eos, max_len))
        f.write(b"".join(struct.pack("<fH", s, len(b)) + b for b, s in m.tokens))
        f.seek(0)
        f.write(struct.pack("<4sI16sIIIIIIIIffIIQQQ", b"l3m\0", 1, m.arch.encode(), m.flags, m.dim, m.n_layers, m.n_heads,
                            m.n_kv_heads, m.ffn_dim, m.vocab, m.ctx, m.rope_theta, m.norm_eps, len(names), 0,
                            toc_offset, tok_offset, 0))
    return {n: len(blobs[n]) for n in names}


def byte_tokens(vocab):
    """256 byte tokens, <s> and </s> (no merges), then empty pieces up to vocab."""
    toks = [(bytes([i]), NO_MERGE) for i in range(256)] + [(b"<s>", NO_MERGE), (b"</s>", NO_MERGE)]
    if vocab < len(toks):
        raise ValueError("vocab must hold 256 bytes plus <s> and </s>")
    return toks + [(b"", NO_MERGE)] * (vocab - len(toks))


def gpt2(dim, n_layers, n_heads, ffn_dim, vocab, ctx, seed=0, std=0.02, stop_tokens=True):
    """A GPT-2-shaped model (LayerNorm with biases, learned positions, GELU MLP, biases on every
    projection, tied head; the reference's "gpt2" arch flags) with N(0, std) weights (std "fan_in":
    1/sqrt(inputs)); norm gains 1 + N(0, 0.1), every bias N(0, 0.02). Drawn in this order: embed,
    pos_embed, norm, norm_b, then per layer attn_norm, attn_norm_b, ffn_norm, ffn_norm_b, wq, wk, wv,
    bq, bk, bv, wo, bo, w_up, b_up, w_down, b_down."""
    rng = np.random.default_rng(seed)
    m = Model("gpt2", LAYERNORM | LEARNED_POS | GELU | TIED, dim, n_layers, n_heads, n_heads, ffn_dim, vocab, ctx, 10000.0, 1e-5)

    def mat(rows, cols):
        scale = np.float32(1 / np.sqrt(cols)) if std == "fan_in" else np.float32(std)
        return (rng.standard_normal((rows, cols), dtype=np.float32) * scale).astype(np.float32)

    def gain(n):
        return (1 + rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32)

    def bias(n):
        return (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    t = m.tensors
    t["embed"] = mat(vocab, dim)
    t["pos_embed"] = mat(ctx, dim)
    t["norm"], t["norm_b"] = gain(dim), bias(dim)
    for i in range(n_layers):
        b = f"blk.{i}."
        t[b + "attn_norm"], t[b + "attn_norm_b"] = gain(dim), bias(dim)
        t[b + "ffn_norm"], t[b + "ffn_norm_b"] = gain(dim), bias(dim)
        t[b + "wq"], t[b + "wk"], t[b + "wv"] = mat(dim, dim), mat(dim, dim), mat(dim, dim)
        t[b + "bq"], t[b + "bk"], t[b + "bv"] = bias(dim), bias(dim), bias(dim)
        t[b + "wo"], t[b + "bo"] = mat(dim, dim), bias(dim)
        t[b + "w_up"], t[b + "b_up"] = mat(ffn_dim, dim), bias(ffn_dim)
        t[b + "w_down"], t[b + "b_down"] = mat(dim, ffn_dim), bias(dim)
    m.tokens = byte_tokens(vocab)
    m.bos, m.eos = (256, 257) if stop_tokens else (-1, -1)
    return m


def llama(dim, n_layers, n_heads, n_kv_heads, ffn_dim, vocab, ctx, theta=10000.0, tied=True, seed=0, std=0.02,
          stop_tokens=True):
    """A Llama-shaped model with N(0, std) weights (std "fan_in": 1/sqrt(inputs)) drawn in this order:
    embed, [lm_head], then per layer wq, wk, wv, wo, w_gate, w_up, w_down. Norm gains are 1.0. With
    stop_tokens False, bos and eos are -1, so a greedy stream never stops early."""
    rng = np.random.default_rng(seed)
    kvd = dim // n_heads * n_kv_heads
    m = Model("llama", TIED if tied else 0, dim, n_layers, n_heads, n_kv_heads, ffn_dim, vocab, ctx, float(theta), 1e-5)

    def mat(rows, cols):
        scale = np.float32(1 / np.sqrt(cols)) if std == "fan_in" else np.float32(std)
        return (rng.standard_normal((rows, cols), dtype=np.float32) * scale).astype(np.float32)

    t = m.tensors
    t["embed"] = mat(vocab, dim)
    if not tied:
        t["lm_head"] = mat(vocab, dim)
    t["norm"] = np.ones(dim, np.float32)
    for i in range(n_layers):
        b = f"blk.{i}."
        t[b + "attn_norm"] = np.ones(dim, np.float32)
        t[b + "ffn_norm"] = np.ones(dim, np.float32)
        t[b + "wq"], t[b + "wk"], t[b + "wv"], t[b + "wo"] = mat(dim, dim), mat(kvd, dim), mat(kvd, dim), mat(dim, dim)
        t[b + "w_gate"], t[b + "w_up"], t[b + "w_down"] = mat(ffn_dim, dim), mat(ffn_dim, dim), mat(dim, ffn_dim)
    m.tokens = byte_tokens(vocab)
    m.bos, m.eos = (256, 257) if stop_tokens else (-1, -1)
    return m


# The benchmark configurations (BASELINE.json "configs"): name -> (shape kwargs, body dtype, head dtype, run ctx).
CONFIGS = {
    "stories15M-bf16": (dict(dim=288, n_layers=6, n_heads=6, n_kv_heads=6, ffn_dim=768, vocab=32000, ctx=256), "bf16", "bf16", 256),
    "stories42M-q8_0": (dict(dim=512, n_layers=8, n_heads=8, n_kv_heads=8, ffn_dim=1376, vocab=32000, ctx=1024), "q8_0", "q8_0", 1024),
    "stories110M-q4_0": (dict(dim=768, n_layers=12, n_heads=12, n_kv_heads=12, ffn_dim=2048, vocab=32000, ctx=1024), "q4_0", "q4_0", 128),
    "SmolLM2-135M-q8_0": (dict(dim=576, n_layers=30, n_heads=9, n_kv_heads=3, ffn_dim=1536, vocab=49152, ctx=2048, theta=100000.0),
                          "q8_0", "q8_0", 256),
    "SmolLM2-135M-mxfp4": (dict(dim=576, n_layers=30, n_heads=9, n_kv_heads=3, ffn_dim=1536, vocab=49152, ctx=2048, theta=100000.0),
                           "mxfp4", "mxfp4", 256),
}


def prompt(n=4, seed=1, vocab=32000):
    """The benchmark prompt: n ids uniform in [0, vocab) from default_rng(seed)."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def make(name, out_dir, ctx=None, stop_tokens=False, seed=0):
    """Write the named configuration to out_dir/<name>.l3m (cached by name, ctx and stop tokens).
    ctx overrides the header context (a 256-step greedy stream after a 4-token prompt needs 260)."""
    shape, dtype, head_dtype, _ = CONFIGS[name]
    shape = dict(shape)
    if ctx:
        shape["ctx"] = ctx
    out = Path(out_dir) / f"{name}-ctx{shape['ctx']}{'-stop' if stop_tokens else ''}-s{seed}.l3m"
    if not out.exists():
        # Several processes (the ranks of one job) may build the same file at once: each writes its own
        # temporary file and moves it into place atomically (the contents are identical).
        out.parent.mkdir(parents=True, exist_ok=True)
        tmp = out.with_suffix(f".{os.getpid()}.tmp")
        write(llama(**shape, seed=seed, stop_tokens=stop_tokens), dtype, head_dtype, tmp)
        os.replace(tmp, out)
    return out


def weight_bytes(name):
    """Algorithmic weight bytes streamed per token: every layer matrix and the head, once."""
    shape, dtype, head_dtype, _ = CONFIGS[name]
    per = {"f32": 4.0, "bf16": 2.0, "q8_0": 34 / 32, "q4_0": 18 / 32, "mxfp4": 17 / 32}
    d, f, L, V = shape["dim"], shape["ffn_dim"], shape["n_layers"], shape["vocab"]
    kvd = d // shape["n_heads"] * shape["n_kv_heads"]
    layer = d * d * 2 + 2 * kvd * d + 3 * f * d
    return int(L * layer * per[dtype] + V * d * per[head_dtype])
