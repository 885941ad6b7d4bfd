"""The oracle, pinned: against the reference's golden vectors and fixtures (tests/golden, made by
make_golden.py from the reference itself), and, where the compiled reference is present
(oracle/_ref), against it function by function, bit for bit."""
import ctypes as C
import hashlib
import json

import numpy as np
import pytest

from conftest import DTYPES, GOLDEN, ORACLE_DIR, VARIANTS, P, OracleRun, Vec
from l3m_b200 import synth

GG = json.loads((GOLDEN / "ggml.json").read_text())
MJ = json.loads((GOLDEN / "models.json").read_text())
ENGINE = np.load(GOLDEN / "engine.npz")
REF_SO = ORACLE_DIR / "_ref" / "libl3m_all.so"


# ---- the on-disk blocks the kernels read

@pytest.mark.parametrize("case", range(6))
def test_quantisers_match_ggml_golden(case):
    """Block bytes for the reference's known-answer inputs (reference tests/unit/test_export.py:37-47)."""
    c = GG["blocks"][case]
    x = np.array(GG[c["input"]], dtype=np.float32)
    assert getattr(synth, c["dtype"])(x).tobytes().hex() == c["hex"]


def test_bf16_and_q8_rounding_golden():
    """bf16 round-to-nearest-even and ggml's x*(1/d) rounding (reference test_export.py:19-22, 50-59)."""
    x = np.array(GG["bf16_in"], dtype=np.float32)
    got = (synth.to_bf16(x).astype(np.uint32) << 16).view(np.float32)
    assert got.tolist() == GG["bf16_out"]
    q = synth.q8_0(np.array(GG["q8_rounding_in"], dtype=np.float32))[0, 2:].view(np.int8)
    assert q.tolist() == GG["q8_rounding_q"] and q[21] == 75


def test_writer_matches_reference_exporter(models):
    """Our .l3m files are byte-identical to the reference exporter's for the same tensors."""
    for (name, dt), path in models.items():
        assert hashlib.sha256(path.read_bytes()).hexdigest() == MJ["sha256"][f"{name}-{dt}"], (name, dt)


# ---- the oracle engine against the reference engine's recorded output

@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("name", ["gqa", "mha40", "gpt2s"])
@pytest.mark.parametrize("path_kind", ["scalar1", "ref"])
def test_oracle_matches_reference_engine(oracle, models, name, dt, path_kind):
    """Greedy tokens and the logits of every sampled position, bit for bit: the reference's scalar
    table (L3M_ISA=scalar; 1 and 3 cores agree) and its fp32 reference path."""
    run = OracleRun(oracle, models[(name, dt)], MJ["prompt"], MJ["steps"], reference=path_kind == "ref")
    want_t = ENGINE[f"{name}-{dt}-{path_kind}-tokens"].tolist()
    want_l = ENGINE[f"{name}-{dt}-{path_kind}-logits"]
    assert run.tokens == want_t
    assert run.logits.shape == want_l.shape
    assert np.array_equal(run.logits.view(np.uint32), want_l.view(np.uint32))


@pytest.mark.parametrize("variant", sorted(VARIANTS))
@pytest.mark.parametrize("path_kind", ["scalar1", "ref"])
def test_oracle_variants_match_reference_engine(oracle, models, variant, path_kind):
    """The same, on a head dtype other than the body's and on a GPT-2 without q, k, v biases
    (reference tests/integration/test_engine.py:187-201)."""
    name, label = variant
    run = OracleRun(oracle, models[variant], MJ["prompt"], MJ["steps"], reference=path_kind == "ref")
    assert run.tokens == ENGINE[f"{name}-{label}-{path_kind}-tokens"].tolist()
    want_l = ENGINE[f"{name}-{label}-{path_kind}-logits"]
    assert run.logits.shape == want_l.shape
    assert np.array_equal(run.logits.view(np.uint32), want_l.view(np.uint32))


SAMPLED = ((0.8, 7), (1.7, 123))


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("name", ["gqa", "mha40", "gpt2s"])
@pytest.mark.parametrize("path_kind", ["scalar1", "ref"])
def test_oracle_sampling_matches_reference_engine(oracle, models, name, dt, path_kind):
    """Temperature sampling: the reference's token streams (one rank; its fp32 path) for two
    (temperature, seed) pairs, token for token."""
    for temp, seed in SAMPLED:
        run = OracleRun(oracle, models[(name, dt)], MJ["prompt"], MJ["steps"], reference=path_kind == "ref", temperature=temp, seed=seed)
        assert run.tokens == ENGINE[f"{name}-{dt}-{path_kind}-t{temp}-s{seed}-tokens"].tolist(), (temp, seed)


def test_oracle_sampler_edges(oracle):
    """The sampler alone: greedy below temperature 0 and for NaN (no draw), the last index for a NaN
    sum, and the xorshift64* draws of the reference (engine.c:98-101)."""
    lg = np.array([0.5, 2.0, 2.0, -30.0], np.float32)
    st = C.c_uint64(5)
    assert oracle.o_sample(P(lg), 4, 0.0, C.byref(st)) == 1 and st.value == 5
    assert oracle.o_sample(P(lg), 4, float("nan"), C.byref(st)) == 1 and st.value == 5
    lg2 = np.array([1.0, np.nan, 3.0], np.float32)
    assert oracle.o_sample(P(lg2), 3, 1.0, C.byref(st)) == 2 and st.value != 5
    s = 5
    for _ in range(3):
        s ^= s >> 12
        s ^= (s << 25) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 27
    st = C.c_uint64(5)
    zeros = np.zeros(1000, np.float32)                 # kept alive while the C code reads it
    got = [oracle.o_sample(P(zeros), 1000, 1.0, C.byref(st)) for _ in range(3)]
    u = ((s * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF) >> 11
    assert st.value == s and got[2] == int(u / 2**53 * 1000)


# ---- function by function against the compiled reference (when oracle/_ref is present)

@pytest.fixture(scope="module")
def ref():
    if not REF_SO.exists():
        pytest.skip("oracle/_ref not built (make -C oracle ref needs the reference sources)")
    lib = C.CDLL(str(REF_SO))
    lib.l3m_tile_bytes.restype = lib.l3m_row_bytes.restype = C.c_size_t
    return lib


GEMV = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(Vec))


class RefTable(C.Structure):
    _fields_ = [("name", C.c_char_p), ("gemv", GEMV * 5), ("attend", C.c_void_p)]


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def random_rows(rng, dtype, n, k, rb, edge=False):
    """File rows of a dtype with random values; edge: q8 -128 weights and subnormal mxfp4 scales
    (legal values the quantisers never produce; reference tests/test_kernels.c:62-68)."""
    buf = np.zeros((n, rb), np.uint8)
    if dtype == 0:
        buf[:] = rng.standard_normal((n, k)).astype(np.float32).view(np.uint8).reshape(n, -1)
    elif dtype == 1:
        buf[:] = synth.to_bf16(rng.standard_normal((n, k)).astype(np.float32)).view(np.uint8).reshape(n, -1)
    else:
        nb = k // 32
        blk = buf.reshape(n, nb, rb // nb)
        if dtype == 2:
            blk[:, :, :2] = f16(np.abs(rng.standard_normal((n, nb))) * 0.01).view(np.uint8).reshape(n, nb, 2)
            blk[:, :, 2:] = rng.integers(-127, 128, (n, nb, 32)).astype(np.int8).view(np.uint8)
            if edge:
                for b in range(nb):
                    blk[:, b, 2 + b % 32] = 0x80
        elif dtype == 3:
            blk[:, :, :2] = f16(rng.standard_normal((n, nb)) * 0.01).view(np.uint8).reshape(n, nb, 2)
            blk[:, :, 2:] = rng.integers(0, 256, (n, nb, 16))
        else:
            blk[:, :, 0] = rng.integers(118, 131, (n, nb))
            blk[:, :, 1:] = rng.integers(0, 256, (n, nb, 16))
            if edge:
                for r in range(n):
                    blk[r, :, 0] = (r + np.arange(nb)) % 3
    return buf


def pack_both(lib_a, lib_b, dtype, rows, ntiles, k, missing, tb):
    n = ntiles * 16
    a = np.zeros(ntiles * tb, np.uint8)
    b = np.zeros(ntiles * tb, np.uint8)
    for t in range(ntiles):
        ptrs = (C.c_void_p * 16)(*[rows[t * 16 + c].ctypes.data if t * 16 + c < n - missing else None for c in range(16)])
        lib_a.l3m_pack_tile(C.c_void_p(a.ctypes.data + t * tb), dtype, ptrs, k)
        lib_b.o_pack_tile(C.c_void_p(b.ctypes.data + t * tb), dtype, ptrs, k)
    return a, b


@pytest.mark.parametrize("dtype", range(5))
def test_kernels_match_reference_scalar_table(ref, oracle, dtype):
    """Packing, activation prepare and the gemv of every dtype, bit for bit against the reference's
    scalar table, over its own test grid (reference tests/test_kernels.c:178-190)."""
    table = RefTable.in_dll(ref, "l3m_kernels_scalar")
    rng = np.random.default_rng(dtype)
    ks = [2, 18, 34, 288, 1376] if dtype <= 1 else [288, 1376, 3072]
    for k in ks:
        for ntiles in (1, 3, 9):
            for missing in (0, 5, 10, 15):
                for edge in ((False, True) if dtype >= 2 and missing == 5 else (False,)):
                    rb, tb = ref.l3m_row_bytes(dtype, k), ref.l3m_tile_bytes(dtype, k)
                    assert rb == oracle.o_row_bytes(dtype, k) and tb == oracle.o_tile_bytes(dtype, k)
                    rows = random_rows(rng, dtype, ntiles * 16, k, rb, edge)
                    ta, tb_ = pack_both(ref, oracle, dtype, rows, ntiles, k, missing, tb)
                    assert np.array_equal(ta, tb_)
                    x = (rng.standard_normal(k) * 4).astype(np.float32)
                    if edge:
                        x[:min(32, k)] = 0                                   # a zero activation block
                    sa, sb = np.zeros(4 * k + 64, np.uint8), np.zeros(4 * k + 64, np.uint8)
                    va, vb = Vec(), Vec()
                    ref.l3m_vec_prepare(C.byref(va), dtype, P(x), k, P(sa))
                    oracle.o_vec_prepare(C.byref(vb), dtype, P(x), k, P(sb))
                    assert np.array_equal(sa, sb)
                    ya, yb = np.zeros(ntiles * 16, np.float32), np.zeros(ntiles * 16, np.float32)
                    table.gemv[dtype](P(ya), P(ta), ntiles, k, C.byref(va))
                    oracle.o_gemv(dtype, P(yb), P(ta), ntiles, k, C.byref(vb))
                    assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32)), (k, ntiles, missing, edge)


def test_ops_match_reference(ref, oracle):
    """rmsnorm and LayerNorm at every n % 8, RoPE, GELU, SiLU and attention, bit for bit (reference
    src/ops.c)."""
    rng = np.random.default_rng(7)
    for n in list(range(1, 41)) + [288, 512, 576, 768]:
        for _ in range(20):
            x = (rng.standard_normal(n) * rng.uniform(0.01, 3)).astype(np.float32)
            w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
            a, b = np.zeros(n, np.float32), np.zeros(n, np.float32)
            ref.l3m_rmsnorm(P(a), P(x), P(w), n, C.c_float(1e-5))
            oracle.o_rmsnorm(P(b), P(x), P(w), n, C.c_float(1e-5))
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), n
    for hd in (48, 64):
        for pos in (0, 1, 7, 259, 1023):
            v = rng.standard_normal(hd * 9).astype(np.float32)
            a, b = v.copy(), v.copy()
            ref.l3m_rope(P(a), 9, hd, pos, C.c_float(10000.0))
            oracle.o_rope(P(b), 9, hd, pos, C.c_float(10000.0))
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for n in list(range(1, 41)) + [96, 288, 576, 768]:
        for _ in range(20):
            x = (rng.standard_normal(n) * rng.uniform(0.01, 3)).astype(np.float32)
            w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
            bb = (0.02 * rng.standard_normal(n)).astype(np.float32)
            a, b = np.zeros(n, np.float32), np.zeros(n, np.float32)
            ref.l3m_layernorm(P(a), P(x), P(w), P(bb), n, C.c_float(1e-5))
            oracle.o_layernorm(P(b), P(x), P(w), P(bb), n, C.c_float(1e-5))
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), n
    u = (rng.standard_normal(100000) * 3).astype(np.float32)
    a, b = u.copy(), u.copy()
    ref.l3m_gelu(P(a), 100000)
    oracle.o_gelu(P(b), 100000)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    g = (rng.standard_normal(50000) * 4).astype(np.float32)
    h = rng.standard_normal(50000).astype(np.float32)
    a, b = h.copy(), h.copy()
    ref.l3m_silu_mul(P(a), P(g), 50000)
    oracle.o_silu_mul(P(b), P(g), 50000)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for hd in (16, 32, 40, 48, 64):
        for pos in (0, 1, 37, 255):
            for qscale in ((2.0, 40.0) if (hd, pos) == (64, 255) else (2.0,)):
                stride = 3 * hd
                q = (rng.uniform(-1, 1, hd) * qscale).astype(np.float32)
                k = synth.to_bf16(rng.uniform(-1, 1, (pos + 1) * stride).astype(np.float32))
                v = synth.to_bf16(rng.uniform(-1, 1, (pos + 1) * stride).astype(np.float32))
                a, b = np.zeros(hd, np.float32), np.zeros(hd, np.float32)
                ref.l3m_attend(P(a), P(q), P(k), P(v), pos, hd, stride)
                oracle.o_attend(P(b), P(q), P(k), P(v), pos, hd, stride)
                assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (hd, pos, qscale)


@pytest.mark.parametrize("dtype", range(1, 5))
def test_sweep_harness_computes_the_matvec(ref, dtype):
    """The matvec sweep's CPU baseline (oracle/sweep_ref.c) runs the reference's picked kernel table
    over a pool of cores: its y equals one call of that table over every tile, bit for bit."""
    import os
    so = ORACLE_DIR / "_ref" / "libsweep_ref.so"
    if not so.exists():
        pytest.skip("oracle/_ref/libsweep_ref.so not built")
    h = C.CDLL(str(so))
    h.sweep_ref_gemv.restype = C.c_double
    h.sweep_ref_gemv.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.POINTER(C.c_int), C.c_int, C.c_int,
                                 C.POINTER(C.c_char_p)]
    ref.l3m_kernels_pick.restype = C.POINTER(RefTable)
    table = ref.l3m_kernels_pick().contents
    rng = np.random.default_rng(dtype)
    ntiles, k = 13, 288
    tiles = random_rows(rng, dtype, ntiles * 16, k, ref.l3m_row_bytes(dtype, k), False)
    packed = np.zeros(ntiles * ref.l3m_tile_bytes(dtype, k), np.uint8)
    for t in range(ntiles):
        ptrs = (C.c_void_p * 16)(*[tiles[t * 16 + c].ctypes.data for c in range(16)])
        ref.l3m_pack_tile(C.c_void_p(packed.ctypes.data + t * ref.l3m_tile_bytes(dtype, k)), dtype, ptrs, k)
    x = rng.standard_normal(k).astype(np.float32)
    cpus = sorted(os.sched_getaffinity(0))[:3]
    y = np.zeros(ntiles * 16, np.float32)
    name = C.c_char_p()
    ns = h.sweep_ref_gemv(dtype, P(packed), ntiles, k, P(x), P(y), (C.c_int * len(cpus))(*cpus), len(cpus), 2, C.byref(name))
    assert ns > 0 and name.value == table.name
    s, v, want = np.zeros(4 * k + 64, np.uint8), Vec(), np.zeros(ntiles * 16, np.float32)
    ref.l3m_vec_prepare(C.byref(v), dtype, P(x), k, P(s))
    table.gemv[dtype](P(want), P(packed), ntiles, k, C.byref(v))
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
