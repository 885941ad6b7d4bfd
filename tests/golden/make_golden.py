"""Regenerate the golden fixtures in this directory from the reference (fpedd/l3m) itself.

Run where the reference checkout and its compiled library exist (oracle/_ref, built by
oracle/Makefile):  python tests/golden/make_golden.py [REFERENCE_CHECKOUT] [--configs]

  ggml.json       ggml block bytes for the reference's own known-answer inputs (its
                  tests/unit/test_export.py:19-59), recomputed with its exporter and checked
                  against the hex strings in that test file.
  models.json     sha256 of small .l3m files written by the reference's exporter from the same
                  fp32 tensors as l3m_b200.synth builds (the tests' `models` fixture).
  engine.npz      the reference engine's greedy tokens and logits on those files: its scalar
                  kernel table on 1 and 3 cores (L3M_ISA=scalar), and its fp32 reference path;
                  and its sampled tokens (temperature 0.8 seed 7, 1.7 seed 123) on 1 core and
                  on the reference path.
  configs.npz     the five BASELINE configs at full size (l3m_b200.synth.make, the bench's files and
                  workload: the config's context, the bench's 4-token prompt, greedy to the end of the
                  context): the reference's greedy tokens (scalar table, 8 cores: the same logits as
                  one core) and a 16-byte sha256 prefix of every position's fp32 logits row, read in
                  its on_token callback (its l3m_logits holds the position that produced the token)
                  and after the call. `--configs` regenerates only this file.
"""
import ctypes as C
import hashlib
import json
import os
import re
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
_args = [a for a in sys.argv[1:] if not a.startswith("--")]
_ref = _args[0] if _args else os.environ.get("L3M_REF_SRC")
if not _ref:
    sys.exit("usage: make_golden.py <reference checkout> (or set L3M_REF_SRC)")
REF = Path(_ref)
sys.path.insert(0, str(REF / "python"))
sys.path.insert(0, str(ROOT))

from l3m import archs, export  # noqa: E402  (the reference's exporter)

from l3m_b200 import synth  # noqa: E402

PROMPT = [5, 77, 200, 3]
STEPS = 40
SPECS = {   # must match tests/conftest.py `models`
    "gqa": dict(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab=300, ctx=96, tied=False, seed=1),
    "mha40": dict(dim=160, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=96, vocab=320, ctx=96, tied=True, seed=2),
    "gpt2s": dict(arch="gpt2", dim=96, n_layers=2, n_heads=4, ffn_dim=192, vocab=310, ctx=96, seed=3),
}
DTYPES = ["f32", "bf16", "q8_0", "q4_0", "mxfp4"]
# Files beyond one dtype per spec (must match tests/conftest.py `VARIANTS`): a body dtype with another
# head dtype (reference tests/integration/test_engine.py:187-191), and a GPT-2 without q, k, v
# biases (its GPT-Neo case, :194-201). key: (spec, label) -> (body dtype, head dtype, drop qkv biases)
VARIANTS = {
    ("gqa", "q4_0+q8_0"): ("q4_0", "q8_0", False), ("gqa", "mxfp4+q8_0"): ("mxfp4", "q8_0", False),
    ("gqa", "q8_0+bf16"): ("q8_0", "bf16", False), ("gpt2s", "q4_0+q8_0"): ("q4_0", "q8_0", False),
    ("gpt2s", "mxfp4+q8_0"): ("mxfp4", "q8_0", False), ("gpt2s", "q8_0+bf16"): ("q8_0", "bf16", False),
    ("gpt2s", "neo-q8_0"): ("q8_0", "q8_0", True),
}


def ggml_golden():
    src = (REF / "tests/unit/test_export.py").read_text()
    halves = np.arange(-16, 16, dtype=np.float32) / 2
    ties = np.float32([127, 0.49999997, -0.49999997, 0.5, -0.5, 1.5, -2.5] + [0] * 25)
    cases = re.findall(r'\("(q8_0|q4_0|mxfp4)", (HALVES|TIES), "([0-9a-f]+)"\)', src)
    assert len(cases) == 6, cases
    out = {"halves": halves.tolist(), "ties": ties.tolist(), "blocks": []}
    for dtype, which, hexs in cases:
        x = halves if which == "HALVES" else ties
        assert getattr(export, dtype)(x).tobytes().hex() == hexs
        out["blocks"].append({"dtype": dtype, "input": which.lower(), "hex": hexs})
    bf = np.array([1.0, 1 + 2**-8, 1 + 3 * 2**-8, 1 + 2**-7 + 2**-9, -2.5], dtype=np.float32)
    out["bf16_in"] = bf.tolist()
    out["bf16_out"] = ((export.to_bf16(bf).astype(np.uint32) << 16).view(np.float32)).tolist()
    m = re.search(r"def test_q8_0_rounds_like_ggml\(\):.*?x = np.array\(\[(.*?)\], dtype", src, re.S)
    xs = [float(v) for v in m.group(1).replace("\n", " ").split(",")]
    q = export.q8_0(np.array(xs, dtype=np.float32))[0, 2:].view(np.int8)
    assert q[21] == 75
    out["q8_rounding_in"] = xs
    out["q8_rounding_q"] = q.tolist()
    return out


def ref_model(m):
    return archs.Model(m.arch, m.flags, m.dim, m.n_layers, m.n_heads, m.n_kv_heads, m.ffn_dim, m.vocab, m.ctx, m.rope_theta,
                       m.norm_eps, tensors=m.tensors, tokens=m.tokens, bos=m.bos, eos=m.eos)


class Opts(C.Structure):
    _fields_ = [("cpus", C.POINTER(C.c_int)), ("n_cpus", C.c_int), ("ctx", C.c_int), ("reference", C.c_int),
                ("force", C.c_int), ("verbose", C.c_int), ("cold", C.c_int)]


def run_ref(lib, path, cores, reference):
    """Greedy tokens and the logits at every sampling position, by feeding prefixes (the reference
    exposes only the last position's logits)."""
    cb_t = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)
    cpus = (C.c_int * cores)(*range(cores))
    o = Opts(cpus=None if reference else cpus, n_cpus=0 if reference else cores, reference=int(reference), force=1)
    m = lib.l3m_load(os.fsencode(str(path)), C.byref(o))
    assert m
    V = lib.l3m_vocab(m)
    toks = []
    cb = cb_t(lambda t, u: toks.append(t) or 1)
    pr = (C.c_int32 * len(PROMPT))(*PROMPT)
    lib.l3m_generate(m, pr, len(PROMPT), STEPS, 0.0, 0, cb, None)
    logits = []
    for i in range(len(toks) + 1):
        seq = PROMPT + toks[:i]
        pr = (C.c_int32 * len(seq))(*seq)
        lib.l3m_generate(m, pr, len(seq), 0, 0.0, 0, cb_t(lambda t, u: 1), None)
        logits.append(np.ctypeslib.as_array(lib.l3m_logits(m), shape=(V,)).copy())
    lib.l3m_free(m)
    return toks, np.stack(logits)


SAMPLED = ((0.8, 7), (1.7, 123))                 # (temperature, seed) of the sampled golden runs


def run_ref_sampled(lib, path, cores, reference, temp, seed):
    """Tokens of one sampled generation (the reference's sampler; one core = one rank)."""
    cb_t = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)
    cpus = (C.c_int * cores)(*range(cores))
    o = Opts(cpus=None if reference else cpus, n_cpus=0 if reference else cores, reference=int(reference), force=1)
    m = lib.l3m_load(os.fsencode(str(path)), C.byref(o))
    assert m
    toks = []
    cb = cb_t(lambda t, u: toks.append(t) or 1)
    pr = (C.c_int32 * len(PROMPT))(*PROMPT)
    lib.l3m_generate(m, pr, len(PROMPT), STEPS, temp, seed, cb, None)
    lib.l3m_free(m)
    return toks


def row_digest(row):
    """The first 16 bytes of the sha256 of one fp32 logits row (little-endian floats)."""
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(row, dtype="<f4").tobytes()).digest()[:16], np.uint8)


def config_streams(lib, cores=8):
    """Greedy token stream and per-position logits digests of the reference on each BASELINE config."""
    out = {}
    cb_t = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)
    prompt = synth.prompt(4, seed=1, vocab=32000)
    with tempfile.TemporaryDirectory() as tmp:
        for name, (_, _, _, ctx) in synth.CONFIGS.items():
            path = synth.make(name, tmp)
            cpus = (C.c_int * cores)(*range(cores))
            m = lib.l3m_load(os.fsencode(str(path)), C.byref(Opts(cpus=cpus, n_cpus=cores, ctx=ctx, force=1)))
            assert m
            V = lib.l3m_vocab(m)
            toks, dig = [], []
            cb = cb_t(lambda t, u: toks.append(t) or dig.append(row_digest(np.ctypeslib.as_array(lib.l3m_logits(m), shape=(V,)))) or 1)
            pr = (C.c_int32 * len(prompt))(*prompt)
            lib.l3m_generate(m, pr, len(prompt), ctx - len(prompt), 0.0, 0, cb, None)
            dig.append(row_digest(np.ctypeslib.as_array(lib.l3m_logits(m), shape=(V,))))
            lib.l3m_free(m)
            out[f"{name}-tokens"] = np.array(toks, np.int32)
            out[f"{name}-digests"] = np.stack(dig)
            print(name, len(toks), "tokens")
    return out


def ref_lib():
    os.environ["L3M_ISA"] = "scalar"
    lib = C.CDLL(str(ROOT / "oracle/_ref/libl3m.so"))
    lib.l3m_load.restype, lib.l3m_load.argtypes = C.c_void_p, [C.c_char_p, C.POINTER(Opts)]
    lib.l3m_generate.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_int, C.c_float, C.c_uint64, C.c_void_p, C.c_void_p]
    lib.l3m_logits.restype, lib.l3m_logits.argtypes = C.POINTER(C.c_float), [C.c_void_p]
    lib.l3m_vocab.argtypes = lib.l3m_free.argtypes = [C.c_void_p]
    return lib


def main():
    if "--configs" in sys.argv:
        np.savez_compressed(HERE / "configs.npz", **config_streams(ref_lib()))
        return
    (HERE / "ggml.json").write_text(json.dumps(ggml_golden(), indent=1))
    lib = ref_lib()
    hashes, arrays = {}, {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, shape in SPECS.items():
            m = (synth.gpt2 if shape.get("arch") == "gpt2" else synth.llama)(**{k: v for k, v in shape.items() if k != "arch"}, std="fan_in", stop_tokens=False)
            for dt in DTYPES:
                path = Path(tmp) / f"{name}-{dt}.l3m"
                export.write(ref_model(m), dt, dt, path)
                hashes[f"{name}-{dt}"] = hashlib.sha256(path.read_bytes()).hexdigest()
                for label, cores, reference in (("scalar1", 1, 0), ("scalar3", 3, 0), ("ref", 1, 1)):
                    toks, lg = run_ref(lib, path, cores, reference)
                    arrays[f"{name}-{dt}-{label}-tokens"] = np.array(toks, np.int32)
                    arrays[f"{name}-{dt}-{label}-logits"] = lg
                for label, cores, reference in (("scalar1", 1, 0), ("ref", 1, 1)):
                    for temp, seed in SAMPLED:
                        toks = run_ref_sampled(lib, path, cores, reference, temp, seed)
                        arrays[f"{name}-{dt}-{label}-t{temp}-s{seed}-tokens"] = np.array(toks, np.int32)
                assert np.array_equal(arrays[f"{name}-{dt}-scalar1-logits"], arrays[f"{name}-{dt}-scalar3-logits"])
                del arrays[f"{name}-{dt}-scalar3-logits"], arrays[f"{name}-{dt}-scalar3-tokens"]
            for (spec, label), (body, head, no_qkv_bias) in VARIANTS.items():
                if spec != name:
                    continue
                v = ref_model(m)
                if no_qkv_bias:
                    v.tensors = {k: t for k, t in m.tensors.items() if not re.fullmatch(r"blk\.\d+\.b[qkv]", k)}
                path = Path(tmp) / f"{name}-{label}.l3m"
                export.write(v, body, head, path)
                hashes[f"{name}-{label}"] = hashlib.sha256(path.read_bytes()).hexdigest()
                for lab, cores, reference in (("scalar1", 1, 0), ("ref", 1, 1)):
                    toks, lg = run_ref(lib, path, cores, reference)
                    arrays[f"{name}-{label}-{lab}-tokens"] = np.array(toks, np.int32)
                    arrays[f"{name}-{label}-{lab}-logits"] = lg
    (HERE / "models.json").write_text(json.dumps({"prompt": PROMPT, "steps": STEPS, "sha256": hashes}, indent=1))
    np.savez_compressed(HERE / "engine.npz", **arrays)
    np.savez_compressed(HERE / "configs.npz", **config_streams(lib))
    print("wrote", ", ".join(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
