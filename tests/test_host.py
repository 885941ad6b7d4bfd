"""Host side of the library, no GPU: the exported C ABI, tile packing and activation prepare
against the oracle, the loader's validation messages (the reference's robustness cases,
tests/integration/test_robustness.py:23-46), GPU-list parsing, and the tokenizer (its tests,
tests/unit/test_tokenizer.py), through a small harness linked against the loader and tokenizer."""
import ctypes as C
import re
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, P, Vec
from l3m_b200 import synth
from test_oracle import random_rows

LIB = ROOT / "l3m_b200" / "libl3m.so"


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "l3m_b200")], check=True)
    import l3m_b200
    return l3m_b200.lib()


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"#define L3M_API.*", "", h.read_text())
        for decl in re.findall(r"L3M_API[^;]*?;", text, re.S):
            fn = re.findall(r"\b(l3m_\w+)\s*\(", decl)
            if fn:
                names.add(fn[0])                                      # a function: the name before (
            else:
                names.update(re.findall(r"\b(l3m_\w+)\s*(?:,|;)", decl))   # data: the declarators
    return names


def test_device_entries_refuse_bad_arguments(lib):
    """Every *_dev entry checks its arguments before touching the GPU: -1 and a message from
    l3m_cuda_error for a wrong dtype, size or missing pointer (no GPU needed)."""
    v, buf = Vec(), (C.c_char * 64)()
    y, t = C.cast(buf, C.c_void_p), C.cast(buf, C.c_void_p)
    cases = [
        (lambda: lib.l3m_gemv_dev(1, 7, y, t, 1, 32, C.byref(v), None), "bad arguments"),
        (lambda: lib.l3m_gemv_dev(1, 2, y, t, 1, 48, C.byref(v), None), "multiple of 32"),
        (lambda: lib.l3m_gemv_dev(1, 1, y, t, 1, 33, C.byref(v), None), "even"),
        (lambda: lib.l3m_gemv_dev(1, 2, y, t, 1, 32, None, None), "required"),
        (lambda: lib.l3m_gemv_splitk_dev(1, y, t, 1, 32, C.byref(v), None), "quantised dtypes only"),
        (lambda: lib.l3m_gemv_splitk_dev(2, y, t, 1, 48, C.byref(v), None), "bad arguments"),
        (lambda: lib.l3m_gemv_splitk_dev(2, y, t, 2049, 512, C.byref(v), None), "exceed the static scratch"),
        (lambda: lib.l3m_gemv_splitk_dev(2, y, t, 1, 32, C.byref(v), None), "required"),
        (lambda: lib.l3m_gemv_splitk_dev(2, y, t, 1, 32, None, None), "required"),
    ]
    p = y
    cases += [
        (lambda: lib.l3m_vec_prepare_dev(9, C.byref(v), p, 32, p, None), "bad arguments"),
        (lambda: lib.l3m_vec_prepare_dev(2, C.byref(v), p, 0, p, None), "bad arguments"),
        (lambda: lib.l3m_vec_prepare_dev(2, C.byref(v), p, 40, p, None), "multiple of 32"),
        (lambda: lib.l3m_vec_prepare_dev(2, C.byref(v), p, 32, None, None), "required"),
        (lambda: lib.l3m_vec_prepare_dev(1, None, p, 32, p, None), "required"),
        (lambda: lib.l3m_block_dots_dev(1, p, t, 1, 32, C.byref(v), None), "quantised dtypes"),
        (lambda: lib.l3m_block_dots_dev(2, p, t, -1, 32, C.byref(v), None), "ntiles >= 0"),
        (lambda: lib.l3m_block_dots_dev(2, p, t, 1, 32, C.byref(v), None), "required"),
        (lambda: lib.l3m_unpack_dev(4, p, p, t, 1, 0, None), "positive multiple of 32"),
        (lambda: lib.l3m_unpack_dev(3, None, p, t, 1, 32, None), "required"),
        (lambda: lib.l3m_attend_dev(p, p, p, p, 0, 12, 12, None), "bad arguments"),
        (lambda: lib.l3m_attend_dev(p, p, None, p, 0, 16, 16, None), "required"),
        (lambda: lib.l3m_sample_dev(p, 0, 1.0, p, p, p, None), "vocab > 0"),
        (lambda: lib.l3m_sample_dev(p, 10, 0.0, p, p, p, None), "temperature > 0"),
        (lambda: lib.l3m_sample_dev(p, 10, 1.0, None, p, p, None), "required"),
        (lambda: lib.l3m_expf_dev(None, p, 5, None), "bad arguments"),
        (lambda: lib.l3m_expf_dev(p, p, -1, None), "bad arguments"),
        (lambda: lib.l3m_chain_cycles_dev(8, C.byref(C.c_double())), "bad arguments"),
    ]
    for call, text in cases:
        assert call() == -1
        assert text in lib.l3m_cuda_error().decode(), text
    assert lib.l3m_gemv_dev(1, 2, y, t, 0, 32, C.byref(v), None) == 0        # nothing to do
    assert lib.l3m_gemv_splitk_dev(2, y, t, 0, 32, C.byref(v), None) == 0
    assert lib.l3m_block_dots_dev(2, p, t, 0, 32, C.byref(v), None) == 0


def test_host_table_fails_loudly_without_a_gpu(lib, capfd):
    """The kernel table's void entries (the reference's l3m_gemv_fn contract) cannot return an error:
    when the device is unusable they say why on stderr and fill the output with NaN."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the failure path is not reached")
    import l3m_b200
    table = l3m_b200.kernels("sm100a")
    k, ntiles = 64, 2
    tiles = np.zeros(ntiles * lib.l3m_tile_bytes(2, k), np.uint8)
    x = np.ones(k, np.float32)
    scratch, v = np.zeros(4 * k + 64, np.uint8), Vec()
    lib.l3m_vec_prepare(C.byref(v), 2, P(x), k, P(scratch))
    y = np.zeros(ntiles * 16, np.float32)
    table.gemv[2](P(y), P(tiles), ntiles, k, C.byref(v))
    assert np.isnan(y).all()
    q, kv, out = np.ones(16, np.float32), np.zeros(64, np.uint16), np.zeros(16, np.float32)
    table.attend(P(out), P(q), P(kv), P(kv), 1, 16, 16)
    assert np.isnan(out).all()
    err = capfd.readouterr().err
    assert "l3m: gemv:" in err and "l3m: attend:" in err


def test_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines()}
    declared = declared_symbols()
    assert len(declared) >= 30
    missing = declared - exported
    assert not missing, missing
    assert not any(s.startswith("o_") for s in exported)   # nothing of the oracle is in the product


@pytest.mark.parametrize("dtype", range(5))
def test_host_layout_matches_oracle(lib, oracle, dtype):
    rng = np.random.default_rng(dtype)
    for k in ([2, 18, 288] if dtype <= 1 else [32, 288, 1376]):
        rb, tb = lib.l3m_row_bytes(dtype, k), lib.l3m_tile_bytes(dtype, k)
        assert (rb, tb) == (oracle.o_row_bytes(dtype, k), oracle.o_tile_bytes(dtype, k))
        rows = random_rows(rng, dtype, 16, k, rb, edge=dtype >= 2)
        ptrs = (C.c_void_p * 16)(*[rows[c].ctypes.data if c < 11 else None for c in range(16)])
        a, b = np.zeros(tb, np.uint8), np.zeros(tb, np.uint8)
        lib.l3m_pack_tile(P(a), dtype, ptrs, k)
        oracle.o_pack_tile(P(b), dtype, ptrs, k)
        assert np.array_equal(a, b)
        da, db = np.zeros(k, np.float32), np.zeros(k, np.float32)
        lib.l3m_dequant_row(P(da), dtype, P(rows[0]), k)
        oracle.o_dequant_row(P(db), dtype, P(rows[0]), k)
        assert np.array_equal(da.view(np.uint32), db.view(np.uint32))
        if dtype >= 1 and k % 32 == 0 or dtype == 1:
            x = (rng.standard_normal(k) * 3).astype(np.float32)
            sa, sb = np.zeros(4 * k + 64, np.uint8), np.zeros(4 * k + 64, np.uint8)
            lib.l3m_vec_prepare(C.byref(Vec()), dtype, P(x), k, P(sa))
            oracle.o_vec_prepare(C.byref(Vec()), dtype, P(x), k, P(sb))
            assert np.array_equal(sa, sb)


def test_parse_cpus(lib):
    buf = (C.c_int * 8)()
    assert lib.l3m_parse_cpus(b"0-3,6", buf, 8) == 5 and list(buf[:5]) == [0, 1, 2, 3, 6]
    for bad in (b"", b"0,", b"3-1", b"a", b"0-9"):
        assert lib.l3m_parse_cpus(bad, buf, 8) == -1, bad


# ---- loader validation, in a child process so the library's stderr can be read

def toc(data):
    n, _, off, _ = struct.unpack_from("<IIQQ", data, 64)
    return {bytes(data[e:e + 64]).split(b"\0")[0].decode(): e for e in range(off, off + 120 * n, 120)}


def patched(src, dst, edits):
    b = bytearray(Path(src).read_bytes())
    base = toc(b) | {"tok": struct.unpack_from("<Q", b, 80)[0]}
    for fmt, where, v in edits:
        struct.pack_into(fmt, b, base[where[0]] + where[1] if isinstance(where, tuple) else where, v)
    Path(dst).write_bytes(b)
    return dst


CASES = {   # header: n_heads at 36, vocab 48, n_tensors 64, toc 72, chat 88 (reference test_robustness.py:23-38)
    "n_tensors": ([("<I", 64, 0xFFFFFFFF)], "truncated file"),
    "toc_offset": ([("<Q", 72, 1 << 63)], "truncated file"),
    "heads": ([("<I", 36, 3)], "bad config"),
    "dtype": ([("<I", ("blk.0.w_up", 64), 9)], "bad dtype"),
    "shape": ([("<Q", ("blk.0.wk", 72), 1)], "nbytes does not match"),
    "offset": ([("<Q", ("blk.0.wq", 104), 1)], "misaligned"),
    "offset_wrap": ([("<Q", ("blk.0.wq", 104), (1 << 64) - 64)], "past the end"),
    "missing": ([("<2s", ("blk.1.w_down", 0), b"zz")], "blk.1.w_down missing"),
    "norm_dtype": ([("<I", ("norm", 64), 1), ("<Q", ("norm", 112), 128)], "tensor norm: expected f32"),
    "tok_count": ([("<I", ("tok", 0), 0x7FFFFFFF)], "bad tokenizer"),
    "tok_len": ([("<H", ("tok", 20), 65535)], "bad tokenizer"),
    "tok_bos": ([("<i", ("tok", 4), 99999)], "bad tokenizer"),
    "tok_vocab": ([("<I", 48, 100)], "tensor embed: expected"),
    "chat_offset": ([("<Q", 88, 1 << 40)], "bad chat section"),
}

LOAD = """
import ctypes as C, sys
sys.path.insert(0, {root!r})
import l3m_b200
lib = l3m_b200.lib()
m = lib.l3m_load({path!r}.encode(), None)
sys.exit(0 if m else 1)
"""


def load_stderr(path):
    r = subprocess.run([sys.executable, "-c", LOAD.format(root=str(ROOT), path=str(path))], capture_output=True, text=True, timeout=120)
    return r.returncode, r.stderr


@pytest.mark.parametrize("case", CASES)
def test_malformed_file_is_a_clean_error(lib, models, tmp_path, case):
    edits, msg = CASES[case]
    path = patched(models[("gqa", "q4_0")], tmp_path / f"{case}.l3m", edits)
    rc, err = load_stderr(path)
    assert rc == 1 and msg in err, err


def test_qkv_biases_come_together(lib, tmp_path):
    m = synth.llama(64, 2, 4, 4, 128, 260, 64, seed=3)
    m.tensors["blk.1.bq"] = np.zeros(64, np.float32)
    synth.write(m, "f32", "f32", tmp_path / "bq.l3m")
    rc, err = load_stderr(tmp_path / "bq.l3m")
    assert rc == 1 and "come together" in err, err


def test_truncated_file(lib, models, tmp_path):
    data = Path(models[("gqa", "q8_0")]).read_bytes()
    toc_off, tok_off = struct.unpack_from("<QQ", data, 72)
    for cut in (0, 100, 1024, toc_off + 10, tok_off + 3, len(data) - 1):
        p = tmp_path / f"cut{cut}.l3m"
        p.write_bytes(data[:cut])
        rc, err = load_stderr(p)
        assert rc == 1 and err.startswith("l3m: "), (cut, err)


# ---- tokenizer, through a harness linked against the loader and tokenizer objects

HARNESS = r"""
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "file.h"
int main(int argc, char **argv) {   /* file, add_bos, then one text per line on stdin: ids out */
    l3m_file f;
    if (l3m_file_open(&f, argv[1])) return 1;
    static char line[1 << 22];
    static int32_t out[1 << 22];
    while (fgets(line, sizeof line, stdin)) {
        size_t n = strlen(line);
        if (n && line[n - 1] == '\n') line[--n] = 0;
        for (size_t i = 0; i < n; i++) if (line[i] == 1) line[i] = '\n';   /* \x01 stands for a newline */
        int k = l3m_tokenizer_encode(&f.tok, line, atoi(argv[2]), out, 1 << 22);
        for (int i = 0; i < k; i++) printf("%d ", out[i]);
        printf("\n");
    }
    l3m_file_close(&f);
    return 0;
}
"""


@pytest.fixture(scope="module")
def tok_bin(tmp_path_factory):
    d = tmp_path_factory.mktemp("tok")
    (d / "h.c").write_text(HARNESS)
    src = ROOT / "l3m_b200" / "csrc"
    exe = d / "tok"
    subprocess.run(["gcc", "-O2", "-std=c11", "-D_GNU_SOURCE", f"-I{src}", "-o", str(exe), str(d / "h.c"),
                    str(src / "file.c"), str(src / "tokenizer.c"), str(src / "pack.c"), "-lm"], check=True)
    return exe


def encode(exe, path, texts, bos=False):
    inp = "".join(t.replace("\n", "\x01") + "\n" for t in texts)
    r = subprocess.run([str(exe), str(path), str(int(bos))], input=inp.encode(), capture_output=True, check=True)
    return [[int(v) for v in line.split()] for line in r.stdout.decode().splitlines()]


def with_tokens(path, tokens, flags=0):
    m = synth.llama(64, 2, 4, 2, 128, len(tokens), 64, seed=1)
    m.tokens, m.flags = tokens, m.flags | flags
    m.bos, m.eos = 256, 257
    synth.write(m, "f32", "f32", path)
    return path


BYTES = synth.byte_tokens(258)


def test_byte_round_trip(tok_bin, tmp_path):
    p = with_tokens(tmp_path / "b.l3m", BYTES)
    texts = ["Once upon a time, there was a little girl named Lily.", "tabs\tand newlines", "ünïcödé 🐍 bytes"]
    for t, ids in zip(texts, encode(tok_bin, p, texts)):
        assert ids == list(t.encode())
    assert encode(tok_bin, p, ["a"], bos=True)[0] == [256, 97]


def test_byte_level_pieces(tok_bin, tmp_path):
    """Merges stay inside GPT-2 pre-tokenizer pieces (reference test_tokenizer.py:31-39)."""
    for digits in (False, True):
        p = with_tokens(tmp_path / f"bpe{digits}.l3m", BYTES + [(b"\n\n", -1.0), (b"'s", -2.0)], synth.DIGITS if digits else 0)
        got = encode(tok_bin, p, ["a\n\nb", "a\n\n", "it's '", "x='s", "\n\n1"])
        assert got[0] == [97, 10, 10, 98]
        assert got[1] == [97, 258]
        assert got[2] == [105, 116, 259, 32, 39]
        assert got[3] == [120, 61, 39, 115]
        assert got[4] == ([258, 49] if digits else [10, 10, 49])


MERGES = [(b"ab", -3.0), (b"bc", -1.0), (b"xy", -1.0), (b"xyz", -2.0), (b"aa", -4.0), (b" a", -5.0), ("ü".encode(), synth.NO_MERGE), (b",", 0.0)]


def test_merges(tok_bin, tmp_path):
    """Highest score first, leftmost on ties, whole characters, duplicates by score (reference test_tokenizer.py:42-61)."""
    p = with_tokens(tmp_path / "m.l3m", BYTES + MERGES)
    got = encode(tok_bin, p, ["abc", "xyz", "aaa", "üé", ","])
    assert got == [[97, 259], [261], [262, 97], [264, 0xC3, 0xA9], [265]]
    sp = with_tokens(tmp_path / "sp.l3m", BYTES + MERGES, synth.SP_PREFIX)
    got = encode(tok_bin, sp, ["a", "", "b"]) + encode(tok_bin, sp, ["b"], bos=True)
    assert got == [[263], [], [32, 98], [256, 32, 98]]


def test_merges_match_quadratic_reference(tok_bin, tmp_path):
    import random
    p = with_tokens(tmp_path / "q.l3m", BYTES + MERGES)
    vocab = {b: i for i, (b, _) in enumerate(BYTES)} | {b: 258 + i for i, (b, _) in enumerate(MERGES)}
    score = {258 + i: s for i, (_, s) in enumerate(MERGES)}
    rng = random.Random(1)
    texts, wants = [], []
    for _ in range(50):
        text = "".join(rng.choices("abcxyz", k=rng.randrange(1, 300)))
        syms = [bytes([c]) for c in text.encode()]
        while cands := [(score[vocab[a + b]], -i) for i, (a, b) in enumerate(zip(syms, syms[1:])) if a + b in vocab]:
            i = -max(cands)[1]
            syms[i:i + 2] = [syms[i] + syms[i + 1]]
        texts.append(text)
        wants.append([vocab[s] for s in syms])
    assert encode(tok_bin, p, texts) == wants


def reference_encoder(path):
    """The compiled reference's encoder (oracle/_ref, its public l3m_load + l3m_encode on the CPU)."""
    from l3m_b200 import Opts
    so = ROOT / "oracle" / "_ref" / "libl3m.so"
    if not so.exists():
        pytest.skip("oracle/_ref not built (make -C oracle ref needs the reference sources)")
    lib = C.CDLL(str(so))
    lib.l3m_load.restype = C.c_void_p
    lib.l3m_load.argtypes = [C.c_char_p, C.POINTER(Opts)]
    lib.l3m_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.POINTER(C.c_int32), C.c_int]
    lib.l3m_free.argtypes = [C.c_void_p]
    one = (C.c_int * 1)(0)
    m = lib.l3m_load(str(path).encode(), C.byref(Opts(cpus=one, n_cpus=1, force=1)))
    assert m

    def enc(text, bos=False):
        data = text.encode()
        buf = (C.c_int32 * (len(data) + 8))()
        n = lib.l3m_encode(m, data, int(bos), buf, len(buf))
        return list(buf[:n])
    return enc, lambda: lib.l3m_free(m)


@pytest.mark.parametrize("flags", ["bpe", "digits", "sp"])
def test_tokenizer_matches_compiled_reference(tok_bin, tmp_path, flags):
    """The encoder against the reference's own (compiled from its sources) on random texts over
    letters, digits, apostrophes, whitespace runs and UTF-8, with a vocabulary of overlapping merges."""
    import random
    rng = random.Random(7)
    alphabet = "abcxyz 019',.\n\t" + "üé🐍"
    merges = [(b"ab", -3.0), (b"bc", -1.0), (b"xy", -1.0), (b"xyz", -2.0), (b"aa", -4.0), (b" a", -5.0), (b" ab", -2.5),
              (b"\n\n", -1.5), (b"'s", -2.0), (b"01", -0.5), (b" 0", -0.7), (b"  ", -0.2), ("ü".encode(), -9.0),
              ("üé".encode(), -0.1), (b"ab", -0.05), (b"c,", -1.0), (b" x", -0.3)]
    flag = {"bpe": 0, "digits": synth.DIGITS, "sp": synth.SP_PREFIX}[flags]
    p = with_tokens(tmp_path / f"r{flags}.l3m", BYTES + merges, flag)
    texts = ["".join(rng.choices(alphabet, k=rng.randrange(0, 80))) for _ in range(300)]
    texts = [t for t in texts if "\0" not in t]
    enc, close = reference_encoder(p)
    try:
        want = [enc(t) for t in texts] + [enc(t, True) for t in texts[:20]]
    finally:
        close()
    assert encode(tok_bin, p, texts) + encode(tok_bin, p, texts[:20], bos=True) == want


def test_long_piece_is_not_quadratic(tok_bin, tmp_path):
    import time
    p = with_tokens(tmp_path / "l.l3m", BYTES + MERGES)
    t = time.perf_counter()
    assert encode(tok_bin, p, ["a" * (1 << 20)])[0] == [262] * (1 << 19)
    assert time.perf_counter() - t < 10


# ---- the packed section (l3m_write_packed)

REF_LIB = ROOT / "oracle" / "_ref" / "libl3m.so"


def _ref_generate(path, n):
    """Greedy tokens and last logits from the reference's own library (one core), or None."""
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref not built")
    lib = C.CDLL(str(REF_LIB))

    class Opts(C.Structure):
        _fields_ = [("cpus", C.POINTER(C.c_int)), ("n_cpus", C.c_int), ("ctx", C.c_int), ("reference", C.c_int),
                    ("force", C.c_int), ("verbose", C.c_int), ("cold", C.c_int)]
    lib.l3m_load.restype, lib.l3m_load.argtypes = C.c_void_p, [C.c_char_p, C.POINTER(Opts)]
    lib.l3m_generate.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.c_float, C.c_uint64, C.c_void_p, C.c_void_p]
    lib.l3m_logits.restype, lib.l3m_logits.argtypes = C.POINTER(C.c_float), [C.c_void_p]
    lib.l3m_vocab.argtypes = lib.l3m_free.argtypes = [C.c_void_p]
    one = (C.c_int * 1)(0)
    m = lib.l3m_load(str(path).encode(), C.byref(Opts(cpus=one, n_cpus=1, force=1)))
    assert m, f"the reference could not load {path}"
    toks = []
    cb = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)(lambda t, u: toks.append(t) or 1)
    pr = (C.c_int32 * 4)(5, 77, 200, 3)
    lib.l3m_generate(m, pr, 4, n, 0.0, 0, cb, None)
    lg = np.ctypeslib.as_array(lib.l3m_logits(m), shape=(lib.l3m_vocab(m),)).copy()
    lib.l3m_free(m)
    return toks, lg


@pytest.mark.parametrize("name", ["gqa", "gpt2s"])
@pytest.mark.parametrize("dt", ["f32", "q8_0", "mxfp4"])
def test_packed_section_is_v1_compatible(lib, models, tmp_path, name, dt):
    """A file with the packed section still reads as v1: the reference's own loader takes it and
    generates the same tokens and logits; packing it again replaces the section (read back checked
    by the writer itself)."""
    src, dst, again = models[(name, dt)], tmp_path / "packed.l3m", tmp_path / "again.l3m"
    assert lib.l3m_write_packed(str(src).encode(), str(dst).encode()) == 0
    assert dst.stat().st_size > src.stat().st_size
    t0, l0 = _ref_generate(src, 12)
    t1, l1 = _ref_generate(dst, 12)
    assert t0 == t1 and np.array_equal(l0.view(np.uint32), l1.view(np.uint32))
    assert lib.l3m_write_packed(str(dst).encode(), str(again).encode()) == 0
    assert again.stat().st_size > dst.stat().st_size          # the old section stays as dead bytes


def test_packed_writer_refuses_bad_input(lib, tmp_path):
    bad = tmp_path / "bad.l3m"
    bad.write_bytes(b"not a model")
    assert lib.l3m_write_packed(str(bad).encode(), str(tmp_path / "o.l3m").encode()) == -1


# ---- the reference's own Python binding over this library

def reference_checkout():
    """The reference checkout (L3M_REF_SRC, else a `reference` directory beside this repository)."""
    import os
    for cand in (os.environ.get("L3M_REF_SRC"), ROOT.parent / "reference"):
        if cand and (Path(cand) / "python" / "l3m" / "__init__.py").exists():
            return Path(cand)
    return None


def test_reference_binding_binds_this_library():
    """The reference's python/l3m (imported from its checkout, unchanged) finds libl3m.so through
    L3M_LIB, binds every symbol of its signature table (python/l3m/__init__.py:23-50) and drives
    l3m_load: on a host without a B200 the load is refused with the library's message and the
    binding raises its RuntimeError. Its Opts and Perf structures have this library's layout."""
    import os
    ref = reference_checkout()
    if ref is None:
        pytest.skip("the reference checkout is not on this host")
    probe = r"""
import ctypes as C, sys
sys.path.insert(0, sys.argv[1])
import l3m
lib = l3m._lib()
print("LIB", lib._name)
sys.path.insert(0, sys.argv[2])
import l3m_b200
assert C.sizeof(l3m.Opts) == C.sizeof(l3m_b200.Opts) and C.sizeof(l3m.Perf) == C.sizeof(l3m_b200.Perf)
assert [f for f, _ in l3m.Opts._fields_] == [f for f, _ in l3m_b200.Opts._fields_]
assert [f for f, _ in l3m.Perf._fields_] == [f for f, _ in l3m_b200.Perf._fields_]
try:
    l3m.Model(sys.argv[3], force=True)
    print("LOADED")
except RuntimeError as e:
    print("REFUSED", e)
"""
    p = synth.llama(64, 2, 4, 2, 128, 300, 64, seed=1)
    path = Path(os.environ.get("TMPDIR", "/tmp")) / "l3m_binding_probe.l3m"
    synth.write(p, "q8_0", "q8_0", path)
    env = dict(os.environ, L3M_LIB=str(ROOT / "l3m_b200" / "libl3m.so"), CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-c", probe, str(ref / "python"), str(ROOT), str(path)], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert f"LIB {ROOT / 'l3m_b200' / 'libl3m.so'}" in r.stdout
    assert "REFUSED" in r.stdout and "l3m: no CUDA device" in r.stderr, (r.stdout, r.stderr)
