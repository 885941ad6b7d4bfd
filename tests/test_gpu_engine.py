"""The decode engine behind l3m.h on a B200, against the oracle: greedy tokens and the logits of
every sampled position bit for bit, on the engine path (the reference's scalar table) and on the
fp32 reference path (reference=True); plus the generate contract (stops, callbacks, errors)
that the reference's tests/integration/test_engine.py checks."""
import ctypes as C
import json

import numpy as np
import pytest

import l3m_b200
from conftest import DTYPES, GOLDEN, VARIANTS, OracleRun
from l3m_b200 import synth

pytestmark = pytest.mark.gpu
MJ = json.loads((GOLDEN / "models.json").read_text())
PROMPT = MJ["prompt"]


def gpu_run(path, prompt, max_new, **kw):
    """Tokens and the logits behind each one (read inside on_token), then the final logits."""
    m = l3m_b200.Model(path, force=True, **kw)
    rows = []
    toks = m.generate(prompt, max_new, temperature=0, on_token=lambda t: rows.append(m.logits) or True)
    rows.append(m.logits)
    return m, toks, np.stack(rows)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("name", ["gqa", "mha40"])
@pytest.mark.parametrize("reference", [False, True])
def test_logits_bit_exact(gpu, oracle, models, name, dt, reference):
    path = models[(name, dt)]
    want = OracleRun(oracle, path, PROMPT, MJ["steps"], reference=reference)
    m, toks, lg = gpu_run(path, PROMPT, MJ["steps"], reference=reference)
    assert toks == want.tokens
    assert lg.shape == want.logits.shape
    bad = np.nonzero((lg.view(np.uint32) != want.logits.view(np.uint32)).any(axis=1))[0]
    assert bad.size == 0, f"first differing position {bad[0]}, max |diff| {np.abs(lg - want.logits).max()}"


ENGINE = np.load(GOLDEN / "engine.npz")
SAMPLED = ((0.8, 7), (1.7, 123))


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("name", ["gqa", "mha40"])
@pytest.mark.parametrize("reference", [False, True])
def test_sampling_matches_reference(gpu, oracle, models, name, dt, reference):
    """Temperature sampling (reference engine.c:370-384, one rank): the reference's own token streams
    (tests/golden, its 1-core table and its fp32 path) and the oracle's, token for token."""
    path = models[(name, dt)]
    m = l3m_b200.Model(path, force=True, reference=reference)
    for temp, seed in SAMPLED:
        got = m.generate(PROMPT, MJ["steps"], temperature=temp, seed=seed)
        want = OracleRun(oracle, path, PROMPT, MJ["steps"], reference=reference, temperature=temp, seed=seed)
        assert got == want.tokens, (temp, seed)
        label = "ref" if reference else "scalar1"
        assert got == ENGINE[f"{name}-{dt}-{label}-t{temp}-s{seed}-tokens"].tolist(), (temp, seed)


def test_sampler_draws_match_oracle(gpu, oracle):
    """l3m_sample_dev (the device sampler l3m_generate runs) against the oracle's sampler, draw by
    draw with the generator state carried along: random logits at three temperatures; a flat
    distribution with a tail of tiny weights over a 49152 vocabulary, whose double running sum
    rounds (the one-thread fallback); a NaN logit (the last index); a 7-entry vocabulary."""
    import torch
    lib = l3m_b200.lib()
    lib.l3m_sample_dev.restype = C.c_int
    lib.l3m_sample_dev.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    rng = np.random.default_rng(4)
    V = 49152
    flat = np.zeros(V, np.float32)
    flat[rng.integers(0, V, 20000)] = -15.9          # e^-15.9: weights far below the running sum's last bit
    flat[rng.integers(0, V, 5000)] = -11.3
    nan = rng.standard_normal(V).astype(np.float32)
    nan[V // 3] = np.nan
    cases = [(rng.standard_normal(V).astype(np.float32) * 3, t) for t in (0.5, 1.0, 2.0)]
    cases += [(flat, 1.0), (nan, 1.0), (rng.standard_normal(7).astype(np.float32), 0.9)]
    for lg, temp in cases:
        dl = torch.from_numpy(lg).cuda()
        scratch = torch.empty(lg.size, dtype=torch.float32, device="cuda")
        st = torch.tensor([12345], dtype=torch.int64, device="cuda")
        tok = torch.zeros(1, dtype=torch.int32, device="cuda")
        ost = C.c_uint64(12345)
        for _ in range(6):
            assert lib.l3m_sample_dev(C.c_void_p(dl.data_ptr()), lg.size, temp, C.c_void_p(st.data_ptr()), C.c_void_p(tok.data_ptr()),
                                      C.c_void_p(scratch.data_ptr()), None) == 0, lib.l3m_cuda_error()
            torch.cuda.synchronize()
            want = oracle.o_sample(lg.ctypes.data_as(C.c_void_p), lg.size, temp, C.byref(ost))
            assert int(tok.item()) == want, (lg.size, temp)
            assert int(st.item()) & 0xFFFFFFFFFFFFFFFF == ost.value


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("reference", [False, True])
def test_gpt2_family_within_tolerance(gpu, oracle, models, dt, reference):
    """The GPT-2 family (LayerNorm with biases, learned positions, GELU MLP, biases on every
    projection) against the oracle, which equals the reference bit for bit: greedy tokens identical
    and the logits of every sampled position within 1e-4 of the largest |logit| (BASELINE's bar for
    floating point). Not bit for bit: GELU's tanhf is the device's, a few ulp from the host libm's."""
    path = models[("gpt2s", dt)]
    want = OracleRun(oracle, path, PROMPT, MJ["steps"], reference=reference)
    m, toks, lg = gpu_run(path, PROMPT, MJ["steps"], reference=reference)
    assert toks == want.tokens
    assert lg.shape == want.logits.shape
    tol = 1e-4 * np.abs(want.logits).max(axis=1, keepdims=True)
    err = np.abs(lg - want.logits)
    assert (err <= tol).all(), f"max |diff| {err.max()} at position {np.argmax(err.max(axis=1))}"


@pytest.mark.parametrize("name,dt", [("gqa", "q8_0"), ("mha40", "bf16"), ("gpt2s", "q4_0")])
def test_packed_section_loads_the_same(gpu, models, tmp_path, name, dt):
    """l3m_load of a file with the packed section (l3m_write_packed) copies those tiles: the same
    tokens and logits as from the rows."""
    src, dst = models[(name, dt)], tmp_path / "packed.l3m"
    assert l3m_b200.lib().l3m_write_packed(str(src).encode(), str(dst).encode()) == 0
    _, t0, l0 = gpu_run(src, PROMPT, 24)
    _, t1, l1 = gpu_run(dst, PROMPT, 24)
    assert t0 == t1 and np.array_equal(l0.view(np.uint32), l1.view(np.uint32))


def test_cold_matches_warm(gpu, models):
    """cold=True (every token streams its weights from HBM: the copies carry an L2 evict-first
    policy) gives the same tokens and logits (reference test_engine.py:231-237)."""
    path = models[("gqa", "q8_0")]
    _, a, la = gpu_run(path, PROMPT, 24)
    _, b, lb = gpu_run(path, PROMPT, 24, cold=True)
    assert a == b and len(a) == 24
    assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))


def test_cold_flush_is_not_token_time(gpu, models):
    """Cold mode evicts the weights before every position and, as the reference's --cold, leaves the
    flush out of the counters: for this 2-layer model the device time per token stays within 1.5x of a
    warm run's, while the flush (1.5 x L2 streamed per position, about 80 us) would more than double it."""
    path = models[("gqa", "q8_0")]
    out = {}
    for cold in (False, True):
        m = l3m_b200.Model(path, force=True, cold=cold)
        m.generate(PROMPT, 24, temperature=0)
        m.perf()
        m.generate(PROMPT, 24, temperature=0)
        dev = m.device_ns()
        p = m.perf()
        assert p["tokens"] == len(PROMPT) + 24 and dev > 0
        assert 0 <= p["ns_wait"] <= p["ns_token"] and p["ns_compute"] == pytest.approx(p["ns_token"] - p["ns_wait"])
        out[cold] = (dev / p["tokens"], p["ns_token"])
        m.close()
    assert out[True][0] < 1.5 * out[False][0], out


@pytest.mark.parametrize("name,dt", [("gqa", "q8_0"), ("mha40", "q4_0"), ("gpt2s", "mxfp4"), ("gqa", "bf16"), ("mha40", "f32"),
                                     ("gpt2s", "bf16")])
def test_prepared_and_float_exchanges_agree(gpu, models, monkeypatch, name, dt):
    """The attention and gate outputs travel between CTAs either as floats (each receiver prepares
    them) or already prepared by their producer (q8 blocks for quantised wo / down, bf16-rounded or
    plain floats for bf16 / f32 ones): the same tokens and logits."""
    _, t0, l0 = gpu_run(models[(name, dt)], PROMPT, 24)
    monkeypatch.setenv("L3M_FLOAT_EXCHANGES", "1")
    _, t1, l1 = gpu_run(models[(name, dt)], PROMPT, 24)
    assert t0 == t1 and np.array_equal(l0.view(np.uint32), l1.view(np.uint32))


@pytest.mark.parametrize("name,dt", [("gqa", "q4_0"), ("mha40", "q4_0"), ("gqa", "mxfp4"), ("gpt2s", "mxfp4")])
def test_widened_and_file_layouts_agree(gpu, models, monkeypatch, name, dt):
    """q4_0 and mxfp4 matrices multiplied as widened q8_0 tiles (the default where they fit) or in
    their file layout (L3M_NO_WIDEN): the same tokens and logits, bit for bit."""
    _, t0, l0 = gpu_run(models[(name, dt)], PROMPT, 24)
    monkeypatch.setenv("L3M_NO_WIDEN", "1")
    _, t1, l1 = gpu_run(models[(name, dt)], PROMPT, 24)
    assert t0 == t1 and np.array_equal(l0.view(np.uint32), l1.view(np.uint32))


def test_mxfp4_scales_without_an_f16_form(gpu, oracle, tmp_path):
    """An mxfp4 model whose block scales 2^(e-128) have no exact f16 (weights about 2^-30: e < 104)
    keeps its matrices in the mxfp4 layout and stays bit-exact with the oracle."""
    m = synth.llama(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab=300, ctx=96, tied=False, seed=5,
                    std=2.0 ** -30, stop_tokens=False)
    path = tmp_path / "tiny-mxfp4.l3m"
    synth.write(m, "mxfp4", "mxfp4", path)
    want = OracleRun(oracle, path, PROMPT, 16)
    _, toks, lg = gpu_run(path, PROMPT, 16)
    assert toks == want.tokens
    assert np.array_equal(lg.view(np.uint32), want.logits.view(np.uint32))


def test_max_new_zero_gives_prompt_logits(gpu, oracle, models):
    path = models[("gqa", "q8_0")]
    m = l3m_b200.Model(path, force=True)
    assert m.generate(PROMPT, 0, temperature=0) == []
    want = OracleRun(oracle, path, PROMPT, 0)
    assert np.array_equal(m.logits.view(np.uint32), want.logits[0].view(np.uint32))


def test_ctx_limits_generation(gpu, oracle, models):
    """pos + 1 >= ctx stops the stream (reference engine.c:322; test_engine.py:319-324)."""
    path = models[("mha40", "bf16")]
    m = l3m_b200.Model(path, ctx=16, force=True)
    assert m.ctx == 16
    toks = m.generate(PROMPT, 100, temperature=0)
    assert len(toks) == 16 - len(PROMPT)
    want = OracleRun(oracle, path, PROMPT, 100, ctx=16)
    assert toks == want.tokens
    assert np.array_equal(m.logits.view(np.uint32), want.logits[-1].view(np.uint32))
    with pytest.raises(ValueError):
        m.generate([1] * 16, 4, temperature=0)


def test_stops_at_eos_and_bos(gpu, oracle, models, tmp_path):
    """EOS and BOS end the stream and are not returned (reference engine.c:323-324)."""
    path = models[("gqa", "f32")]
    free = OracleRun(oracle, path, PROMPT, 24).tokens
    base = synth.llama(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=128, vocab=300, ctx=96, tied=False, seed=1,
                       std="fan_in", stop_tokens=False)
    for attr in ("eos", "bos"):
        stop = free[8]
        if stop in free[:8]:
            continue
        m = base
        m.bos, m.eos = (-1, stop) if attr == "eos" else (stop, -1)
        p = tmp_path / f"{attr}.l3m"
        synth.write(m, "f32", "f32", p)
        got = l3m_b200.Model(p, force=True).generate(PROMPT, 24, temperature=0)
        assert got == free[:8]
        assert OracleRun(oracle, p, PROMPT, 24).tokens == free[:8]


def test_callback_stops_and_perf_counts(gpu, models):
    """on_token returning False stops after that token (reference test_engine.py:279-287)."""
    m = l3m_b200.Model(models[("gqa", "q8_0")], force=True)
    seen = []
    out = m.generate(PROMPT, 30, temperature=0, on_token=lambda t: seen.append(t) or len(seen) < 5)
    assert out == seen and len(out) == 5
    p = m.perf()
    assert p["tokens"] == len(PROMPT) + len(out) - 1 and p["ns_token"] > 0 and p["bytes_token"] > 0
    assert 0 <= p["ns_wait"] < p["ns_token"]
    assert all(np.isnan(v) for v in m.perf().values())
    full = m.generate(PROMPT, 30, temperature=0)
    assert full[:5] == out


def test_c_api_contracts(gpu, models):
    """What the Python wrapper guards, refused by the C API too (reference test_engine.py:290-302)."""
    m = l3m_b200.Model(models[("gqa", "f32")], ctx=16, force=True)
    lib, h, cb = m._lib, m._ptr, l3m_b200._CB(lambda t, u: 1)
    assert lib.l3m_generate(h, (C.c_int32 * 1)(m.vocab), 1, 2, 0.0, 0, cb, None) == -1
    assert lib.l3m_generate(h, (C.c_int32 * 16)(*[1] * 16), 16, 2, 0.0, 0, cb, None) == 0
    assert lib.l3m_generate(h, (C.c_int32 * 0)(), 0, 2, 0.0, 0, cb, None) == 0
    buf = (C.c_int32 * 3)()
    assert lib.l3m_encode(h, b"hello", 1, buf, 2) == -1
    n = C.c_int(7)
    lib.l3m_decode(h, 99999, C.byref(n))
    assert n.value == 0
    assert lib.l3m_perf_read(h, C.byref(l3m_b200.Perf())) == -1


def test_repeat_generate_is_deterministic(gpu, models):
    m = l3m_b200.Model(models[("mha40", "q4_0")], force=True)
    a = m.generate(PROMPT, 30, temperature=0)
    la = m.logits
    b = m.generate(PROMPT, 30, temperature=0)
    assert a == b and np.array_equal(la.view(np.uint32), m.logits.view(np.uint32))


def test_describe_and_python_api(gpu, models):
    path = models[("gqa", "f32")]
    with l3m_b200.Model(path, force=True, verbose=True) as m:
        assert "GPU" in m.describe() and "sm100a" in m.describe()
        assert m.generate(PROMPT, 3, temperature=0)
    with pytest.raises(ValueError):
        m.describe()
    with pytest.raises(ValueError):
        l3m_b200.Model(path, ctx=1)


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_mixed_head_dtype_and_no_qkv_biases(gpu, oracle, models, variant):
    """A head dtype other than the body's, and a GPT-2 without q, k, v biases (reference
    tests/integration/test_engine.py:187-201), against the oracle (pinned to the reference on the
    same files): Llama bit for bit; the GPT-2 family's logits within 1e-4 of the largest |logit|."""
    path = models[variant]
    want = OracleRun(oracle, path, PROMPT, MJ["steps"])
    _, toks, lg = gpu_run(path, PROMPT, MJ["steps"])
    assert toks == want.tokens and lg.shape == want.logits.shape
    if variant[0] == "gpt2s":
        assert (np.abs(lg - want.logits) <= 1e-4 * np.abs(want.logits).max(axis=1, keepdims=True)).all()
    else:
        assert np.array_equal(lg.view(np.uint32), want.logits.view(np.uint32))


@pytest.mark.parametrize("name,dt", [("gqa", "q8_0"), ("mha40", "mxfp4"), ("gpt2s", "bf16")])
def test_cluster_counts_give_identical_logits(gpu, models, monkeypatch, name, dt):
    """The vocabulary split over one cluster (16 CTAs) and over every cluster the GPU holds gives the
    same tokens and logits (the reference's core-count invariance, test_engine.py:217-228)."""
    _, t0, l0 = gpu_run(models[(name, dt)], PROMPT, 24)
    monkeypatch.setenv("L3M_CLUSTERS", "1")
    _, t1, l1 = gpu_run(models[(name, dt)], PROMPT, 24)
    assert t0 == t1 and np.array_equal(l0.view(np.uint32), l1.view(np.uint32))


def test_api_misuse_raises(gpu, models):
    """Reference tests/integration/test_robustness.py:94-114: bad prompts, an exception from
    on_token, generate or close from on_token, use after close."""
    m = l3m_b200.Model(models[("gqa", "q8_0")], force=True)
    for bad in ([], [-1], [m.vocab], [2**40]):
        with pytest.raises(ValueError):
            m.generate(bad, 2)

    def boom(t):
        raise KeyError("stop")
    with pytest.raises(KeyError):
        m.generate([1], 5, on_token=boom)
    for reenter in (lambda t: m.generate([1], 1), lambda t: m.close()):
        with pytest.raises(RuntimeError):
            m.generate([1], 5, on_token=reenter)
    streamed = []
    out = m.generate([1], 5, on_token=lambda t: streamed.append(m.decode_bytes([t])))
    assert b"".join(streamed) == m.decode_bytes(out)
    m.close()
    m.close()
    for f in (m.describe, lambda: m.generate([1], 2), lambda: m.encode("a")):
        with pytest.raises(ValueError):
            f()


def test_bad_gpu_lists_are_refused(gpu, models):
    """cpus is the GPU ordinal list: a repeated, missing or negative ordinal is a clean error
    (reference test_robustness.py:117-125, for cores)."""
    path = models[("gqa", "f32")]
    for cpus in ([0, 0], [100000], [-1]):
        with pytest.raises(RuntimeError):
            l3m_b200.Model(path, cpus=cpus, force=True)
    assert l3m_b200.Model(path, cpus=[0], force=True).generate(PROMPT, 3, temperature=0)


def test_threads_share_a_model(gpu, models):
    """Calls from several threads are serialised; a close from another thread ends theirs cleanly
    (reference test_robustness.py:128-146)."""
    import contextlib
    import threading
    m = l3m_b200.Model(models[("gpt2s", "bf16")], force=True)
    want, got = m.generate([1, 5], 12, temperature=0), []

    def worker():
        with contextlib.suppress(ValueError):
            for _ in range(5):
                got.append(m.generate([1, 5], 12, temperature=0))

    def together(*fns):
        threads = [threading.Thread(target=f) for f in fns]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
    together(worker, worker, worker)
    assert got == [want] * 15
    together(worker, worker, worker, m.close)
    assert got == [want] * len(got)


def test_model_without_bos(gpu, models):
    """A file whose bos is -1: no BOS in front of an encoded prompt (reference test_robustness.py:81-83)."""
    m = l3m_b200.Model(models[("gqa", "f32")], force=True)
    assert m.bos == -1 and m.encode("ab") == [97, 98]


def test_sampling_distribution(gpu, models):
    """Chi-square of the first sampled token over 2000 seeds against softmax(logits / T)
    (reference test_engine.py:251-265)."""
    m = l3m_b200.Model(models[("gpt2s", "f32")], force=True)
    ids, temp, n = PROMPT[:1], 0.5, 2000
    assert m.generate(ids, 0, temperature=0) == []
    z = m.logits.astype(np.float64) / temp
    p = np.exp(z - z.max())
    p /= p.sum()
    counts = np.zeros(m.vocab)
    for seed in range(n):
        out = m.generate(ids, 1, temperature=temp, seed=seed)
        counts[out[0]] += 1
    big = p * n >= 5
    obs, exp = np.append(counts[big], counts[~big].sum()), np.append(p[big], p[~big].sum()) * n
    df = len(obs) - 1
    assert ((obs - exp) ** 2 / exp).sum() < df + 5 * np.sqrt(2 * df)


def test_load_refuses_over_budget(gpu, tmp_path):
    """Weights larger than the GPU's persisting L2 window are refused unless force (reference
    test_engine.py:112-119): here 160 MiB of f32 against a 126 MB L2."""
    m = synth.llama(dim=512, n_layers=10, n_heads=8, n_kv_heads=8, ffn_dim=2048, vocab=300, ctx=64, seed=4)
    synth.write(m, "f32", "f32", tmp_path / "big.l3m")
    with pytest.raises(RuntimeError):
        l3m_b200.Model(tmp_path / "big.l3m", cpus=[0])
    assert "on 1 GPU " in l3m_b200.Model(tmp_path / "big.l3m", cpus=[0], force=True).describe()
