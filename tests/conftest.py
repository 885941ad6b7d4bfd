"""Shared fixtures. `-m "not gpu"` runs the oracle, format, tokenizer and ABI checks on the CPU;
`-m gpu` runs the parity tests of the CUDA path against the oracle on a B200."""
import copy
import ctypes as C
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from l3m_b200 import synth  # noqa: E402

ORACLE_DIR = ROOT / "oracle"
GOLDEN = ROOT / "tests" / "golden"
DTYPES = ["f32", "bf16", "q8_0", "q4_0", "mxfp4"]
# Files beyond one dtype per model (the same table as tests/golden/make_golden.py): a body dtype with
# another head dtype (reference tests/integration/test_engine.py:187-191) and a GPT-2 without q, k,
# v biases (its GPT-Neo case, :194-201). (model, label) -> (body dtype, head dtype, drop qkv biases)
VARIANTS = {
    ("gqa", "q4_0+q8_0"): ("q4_0", "q8_0", False), ("gqa", "mxfp4+q8_0"): ("mxfp4", "q8_0", False),
    ("gqa", "q8_0+bf16"): ("q8_0", "bf16", False), ("gpt2s", "q4_0+q8_0"): ("q4_0", "q8_0", False),
    ("gpt2s", "mxfp4+q8_0"): ("mxfp4", "q8_0", False), ("gpt2s", "q8_0+bf16"): ("q8_0", "bf16", False),
    ("gpt2s", "neo-q8_0"): ("q8_0", "q8_0", True),
}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


def gpu_available():
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=20)
        return out.returncode == 0 and "GPU" in out.stdout
    except Exception:
        return False


from l3m_b200 import Vec  # noqa: E402  (one ctypes struct for the library and the oracle)


def P(a):
    return C.c_void_p(a.ctypes.data)


@pytest.fixture(scope="session")
def oracle():
    """The CPU oracle (test infrastructure): oracle/liboracle.so, built by oracle/Makefile."""
    return load_oracle()


def load_oracle():
    so = ORACLE_DIR / "liboracle.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "oracle"], check=True)
    lib = C.CDLL(str(so))
    vp, i = C.c_void_p, C.c_int
    sigs = {
        "o_load": (vp, [C.c_char_p, i]), "o_free": (None, [vp]), "o_vocab": (i, [vp]), "o_ctx": (i, [vp]),
        "o_eos": (i, [vp]), "o_bos": (i, [vp]),
        "o_forward": (C.POINTER(C.c_float), [vp, C.c_int32, i, i]),
        "o_generate": (i, [vp, C.POINTER(C.c_int32), i, i, vp, vp, C.POINTER(i), i]),
        "o_generate_t": (i, [vp, C.POINTER(C.c_int32), i, i, C.c_float, C.c_uint64, vp, vp, C.POINTER(i), i]),
        "o_sample": (C.c_int32, [vp, i, C.c_float, C.POINTER(C.c_uint64)]),
        "o_layernorm": (None, [vp, vp, vp, vp, i, C.c_float]),
        "o_gelu": (None, [vp, i]),
        "o_row_bytes": (C.c_size_t, [i, i]), "o_tile_bytes": (C.c_size_t, [i, i]),
        "o_pack_tile": (None, [vp, i, C.POINTER(vp), i]), "o_dequant_row": (None, [vp, i, vp, i]),
        "o_vec_prepare": (None, [C.POINTER(Vec), i, vp, i, vp]),
        "o_gemv": (None, [i, vp, vp, i, i, C.POINTER(Vec)]),
        "o_block_dots": (None, [i, vp, vp, i, i, C.POINTER(Vec)]),
        "o_unpack": (None, [i, vp, vp, vp, i, i]),
        "o_rmsnorm": (None, [vp, vp, vp, i, C.c_float]), "o_rope": (None, [vp, i, i, i, C.c_float]),
        "o_silu_mul": (None, [vp, vp, i]), "o_attend": (None, [vp, vp, vp, vp, i, i, i]),
        "o_expf": (C.c_float, [C.c_float]), "o_expf_n": (None, [C.c_void_p, C.c_void_p, C.c_int]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


class OracleRun:
    """Generate on the oracle (greedy, or sampled at temperature > 0): tokens, logits of every
    sampled position, positions run."""

    def __init__(self, oracle, path, prompt, max_new, ctx=0, reference=False, temperature=0.0, seed=0):
        m = oracle.o_load(os.fsencode(str(path)), ctx)
        assert m, f"oracle could not load {path}"
        try:
            V = oracle.o_vocab(m)
            out = (C.c_int32 * max(max_new, 1))()
            lg = np.zeros((max_new + 1, V), np.float32)
            npos = C.c_int()
            pr = (C.c_int32 * len(prompt))(*prompt)
            n = oracle.o_generate_t(m, pr, len(prompt), max_new, temperature, seed, out, P(lg), C.byref(npos), int(reference))
            self.tokens = list(out[:n])
            self.n_pos = npos.value
            rows = self.n_pos - (len(prompt) - 1)
            self.logits = lg[:rows]
        finally:
            oracle.o_free(m)


def oracle_stream(path, prompt, max_new, ctx):
    """OracleRun's (tokens, logits) for one file, as a picklable call for a spawned worker process
    (spawned, so it inherits no CUDA state): the oracle is single-threaded, and independent runs
    go faster side by side."""
    run = OracleRun(load_oracle(), path, prompt, max_new, ctx=ctx)
    return run.tokens, run.logits


@pytest.fixture(scope="session")
def models(tmp_path_factory):
    """Small seeded models: a GQA Llama with an untied head (head_dim 16), an MHA Llama with a tied
    head (head_dim 40) and a GPT-2 (LayerNorm, learned positions, GELU, biases; head_dim 24), each
    in every dtype, plus the VARIANTS files; weights scaled 1/sqrt(inputs) so activations cover a
    wide range."""
    out = tmp_path_factory.mktemp("models")
    specs = {
        "gqa": dict(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab=300, ctx=96, tied=False, seed=1),
        "mha40": dict(dim=160, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=96, vocab=320, ctx=96, tied=True, seed=2),
        "gpt2s": dict(arch="gpt2", dim=96, n_layers=2, n_heads=4, ffn_dim=192, vocab=310, ctx=96, seed=3),
    }
    paths = {}
    for name, shape in specs.items():
        m = (synth.gpt2 if shape.get("arch") == "gpt2" else synth.llama)(**{k: v for k, v in shape.items() if k != "arch"}, std="fan_in", stop_tokens=False)
        for dt in DTYPES:
            p = out / f"{name}-{dt}.l3m"
            synth.write(m, dt, dt, p)
            paths[(name, dt)] = p
        for (spec, label), (body, head, no_qkv_bias) in VARIANTS.items():
            if spec == name:
                v = copy.copy(m)
                if no_qkv_bias:
                    v.tensors = {k: t for k, t in m.tensors.items() if not re.fullmatch(r"blk\.\d+\.b[qkv]", k)}
                p = out / f"{name}-{label}.l3m"
                synth.write(v, body, head, p)
                paths[(name, label)] = p
    return paths


@pytest.fixture(scope="session")
def gpu():
    if not gpu_available():
        pytest.fail("the gpu tests need a B200 (nvidia-smi finds none); there is no CPU fallback")
    import l3m_b200
    lib = l3m_b200.lib()
    return lib
