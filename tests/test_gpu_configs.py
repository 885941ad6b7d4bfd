"""The BASELINE.json decode configurations at full size on a B200: 256 greedy steps after the
4-token benchmark prompt, tokens identical to the oracle's and the logits of every sampled position
bit-identical (north_star: identical 256-step greedy streams; logits within 1e-4 relative — held
here to 0). Header and run context are 264 so no stream is cut by the context limit."""
import multiprocessing as mp
import os

import numpy as np
import pytest

import l3m_b200
from conftest import oracle_stream
from l3m_b200 import synth

pytestmark = pytest.mark.gpu
STEPS = 256
CTX = 264


PROMPT = synth.prompt(4, seed=1, vocab=32000)


@pytest.fixture(scope="module")
def oracle_streams(tmp_path_factory):
    """Every config's file and its oracle stream (tokens, logits), the oracle runs side by side in
    spawned processes (one after another they take minutes)."""
    model_dir = tmp_path_factory.mktemp("configs")
    paths = {name: synth.make(name, model_dir, ctx=CTX) for name in synth.CONFIGS}
    with mp.get_context("spawn").Pool(max(1, min(len(paths), os.cpu_count() or 1))) as pool:
        jobs = {name: pool.apply_async(oracle_stream, (str(p), PROMPT, STEPS, CTX)) for name, p in paths.items()}
        return {name: (paths[name], *job.get()) for name, job in jobs.items()}


@pytest.mark.parametrize("name", list(synth.CONFIGS))
def test_config_stream_bit_exact(gpu, oracle_streams, name):
    path, want_tokens, want_logits = oracle_streams[name]
    vocab = synth.CONFIGS[name][0]["vocab"]
    prompt = PROMPT
    assert len(want_tokens) == STEPS
    m = l3m_b200.Model(path, ctx=CTX, force=True)
    rows = []
    toks = m.generate(prompt, STEPS, temperature=0, on_token=lambda t: rows.append(m.logits) or True)
    rows.append(m.logits)
    lg = np.stack(rows)
    assert lg.shape == (STEPS + 1, vocab)
    first = next((i for i, (a, b) in enumerate(zip(toks, want_tokens)) if a != b), None)
    if first is not None:
        top2 = np.sort(want_logits[first])[-2:]
        pytest.fail(f"stream departs at step {first}; oracle top-2 gap there {top2[1] - top2[0]:.3g}")
    assert toks == want_tokens
    bad = np.nonzero((lg.view(np.uint32) != want_logits.view(np.uint32)).any(axis=1))[0]
    assert bad.size == 0, f"first differing position {bad[0]}, max |diff| {np.abs(lg - want_logits).max()}"


GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "configs.npz"))


def row_digest(row):
    """tests/golden/make_golden.py's digest: the first 16 bytes of the sha256 of the fp32 row."""
    import hashlib
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(row, dtype="<f4").tobytes()).digest()[:16], np.uint8)


@pytest.mark.parametrize("name", list(synth.CONFIGS))
def test_config_stream_matches_reference_run(gpu, tmp_path_factory, name):
    """Each config at full size and on the bench's own workload (its file, its context, the 4-token
    prompt, greedy to the end of the context) against a recorded run of the reference itself
    (tests/golden/configs.npz: its scalar table's tokens and a digest of every position's logits
    row): the same tokens and every logits row bit-identical."""
    _, _, _, ctx = synth.CONFIGS[name]
    path = synth.make(name, tmp_path_factory.mktemp("bench_files"))
    want_tokens, want_dig = GOLDEN[f"{name}-tokens"].tolist(), GOLDEN[f"{name}-digests"]
    m = l3m_b200.Model(path, ctx=ctx, force=True)
    dig = []
    toks = m.generate(PROMPT, ctx - len(PROMPT), temperature=0, on_token=lambda t: dig.append(row_digest(m.logits)) or True)
    dig.append(row_digest(m.logits))
    m.close()
    assert toks == want_tokens
    got = np.stack(dig)
    assert got.shape == want_dig.shape
    bad = np.nonzero((got != want_dig).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} logits rows differ, the first at position {bad[0]}"
