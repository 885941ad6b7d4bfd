"""The BASELINE.json decode configurations at full size on a B200: 256 greedy steps after the
4-token benchmark prompt, tokens identical to the oracle's and the logits of every sampled position
bit-identical (north_star: identical 256-step greedy streams; logits within 1e-4 relative — held
here to 0). Header and run context are 264 so no stream is cut by the context limit."""
import numpy as np
import pytest

import l3m_b200
from conftest import OracleRun
from l3m_b200 import synth

pytestmark = pytest.mark.gpu
STEPS = 256
CTX = 264


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("configs")


@pytest.mark.parametrize("name", list(synth.CONFIGS))
def test_config_stream_bit_exact(gpu, oracle, model_dir, name):
    path = synth.make(name, model_dir, ctx=CTX)
    vocab = synth.CONFIGS[name][0]["vocab"]
    prompt = synth.prompt(4, seed=1, vocab=32000)
    want = OracleRun(oracle, path, prompt, STEPS, ctx=CTX)
    assert len(want.tokens) == STEPS
    m = l3m_b200.Model(path, ctx=CTX, force=True)
    rows = []
    toks = m.generate(prompt, STEPS, temperature=0, on_token=lambda t: rows.append(m.logits) or True)
    rows.append(m.logits)
    lg = np.stack(rows)
    assert lg.shape == (STEPS + 1, vocab)
    first = next((i for i, (a, b) in enumerate(zip(toks, want.tokens)) if a != b), None)
    if first is not None:
        top2 = np.sort(want.logits[first])[-2:]
        pytest.fail(f"stream departs at step {first}; oracle top-2 gap there {top2[1] - top2[0]:.3g}")
    assert toks == want.tokens
    bad = np.nonzero((lg.view(np.uint32) != want.logits.view(np.uint32)).any(axis=1))[0]
    assert bad.size == 0, f"first differing position {bad[0]}, max |diff| {np.abs(lg - want.logits).max()}"
