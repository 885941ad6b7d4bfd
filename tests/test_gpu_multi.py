"""One model split over several GPUs of one box (the reference's output-channel sharding over
cores, src/engine.c:467-476, 135-152): the reference's invariant that the logits do not depend on
how many ranks share the work (tests/integration/test_engine.py:217-228) must hold for GPUs. Greedy
tokens and every sampled position's logits at 2, 3, 4 and 8 GPUs equal the one-GPU run bit for bit,
on every dtype, on a GQA model whose kv groups straddle GPUs, on the GPT-2 family and on the fp32
reference path; temperature sampling draws the same tokens. Runs on as many GPUs as the box shows
(at least 2); one host thread drives every GPU of a model, as one process drives every core of a
model in the reference."""
import subprocess

import numpy as np
import pytest

import l3m_b200
from l3m_b200 import synth

pytestmark = pytest.mark.gpu

PROMPT = [5, 77, 200, 3]


def visible_gpus():
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=20).stdout
        return sum(1 for line in out.splitlines() if line.startswith("GPU "))
    except Exception:
        return 0


@pytest.fixture(scope="module")
def ngpu(gpu):
    n = visible_gpus()
    if n < 2:
        pytest.skip(f"the split-model tests need at least 2 GPUs; this box shows {n}")
    return n


@pytest.fixture(scope="module")
def wide(tmp_path_factory):
    """A model wide enough for 8 GPUs (16 dim tiles, 32 ffn tiles), 8 heads over 2 kv heads, so that
    kv groups straddle GPUs at 3 and 8."""
    out = tmp_path_factory.mktemp("wide")
    m = synth.llama(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, ffn_dim=512, vocab=500, ctx=96, tied=False, seed=7, std="fan_in",
                    stop_tokens=False)
    paths = {}
    for dt in ("q8_0", "q4_0", "mxfp4", "bf16", "f32"):
        p = out / f"wide-{dt}.l3m"
        synth.write(m, dt, dt, p)
        paths[dt] = p
    return paths


def run(path, cpus, max_new=24, temperature=0.0, seed=0, **kw):
    m = l3m_b200.Model(path, cpus=cpus, force=True, **kw)
    rows = []
    toks = m.generate(PROMPT, max_new, temperature=temperature, seed=seed, on_token=lambda t: rows.append(m.logits) or True)
    rows.append(m.logits)
    m.close()
    return toks, np.stack(rows)


@pytest.mark.parametrize("dt", ["q8_0", "q4_0", "mxfp4", "bf16", "f32"])
def test_split_gives_identical_logits(ngpu, wide, dt):
    t1, l1 = run(wide[dt], [0])
    for n in (2, 3, 4, 8):
        if n > ngpu:
            continue
        tn, ln = run(wide[dt], list(range(n)))
        assert tn == t1, (n, tn, t1)
        assert np.array_equal(ln.view(np.uint32), l1.view(np.uint32)), f"{n} GPUs: logits differ"


def test_split_reference_path_and_sampling(ngpu, wide):
    """The fp32 reference path split the same way; temperature sampling over the whole row gathered
    on every GPU draws what one GPU draws."""
    t1, l1 = run(wide["q8_0"], [0], reference=True)
    t2, l2 = run(wide["q8_0"], [0, 1], reference=True)
    assert t1 == t2 and np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    for seed in (1, 2):
        s1, _ = run(wide["q4_0"], [0], max_new=32, temperature=0.9, seed=seed)
        s2, _ = run(wide["q4_0"], list(range(min(ngpu, 4))), max_new=32, temperature=0.9, seed=seed)
        assert s1 == s2, seed


@pytest.mark.parametrize("name,dt", [("gqa", "q8_0"), ("gpt2s", "bf16"), ("mha40", "mxfp4")])
def test_split_small_models(ngpu, models, name, dt):
    """The shared small models: a GQA model (4 heads over 2 kv heads) at 2 and 3 GPUs, where GPU 1 of
    3 holds a kv head whose group starts on GPU 0; the GPT-2 family; a tied head."""
    t1, l1 = run(models[(name, dt)], [0])
    for n in (2, 3):
        if n > ngpu:
            continue
        tn, ln = run(models[(name, dt)], list(range(n)))
        assert tn == t1 and np.array_equal(ln.view(np.uint32), l1.view(np.uint32)), (name, dt, n)


def test_split_refuses_more_gpus_than_tiles(ngpu, models):
    """dim 64 has 4 tiles: a split over more GPUs than that is refused, not run."""
    if ngpu < 5:
        pytest.skip("needs 5 GPUs")
    with pytest.raises(RuntimeError):
        l3m_b200.Model(models[("gqa", "q8_0")], cpus=list(range(5)), force=True)
