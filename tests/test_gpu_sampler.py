"""Device sampling (qne_sampler_*, qne_step_sample) against the CPU restatement of the reference
sampler (oracle/sampler.py, itself pinned by the reference's unit tests in
tests/test_sampler_oracle.py): the same unit tests through the device, identical token streams
on random full-vocabulary logits for greedy / temperature / top-k / top-p / presence penalty /
mask / tool-call bias settings, error behaviour, and the model-level loop."""
import math

import numpy as np
import pytest
import torch

import qne
from oracle.sampler import Sampler as OracleSampler
from qne import synth

pytestmark = pytest.mark.gpu
VOCAB = 248320


@pytest.fixture(scope="module")
def small(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=512, seed=31)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    yield m
    m.close()


@pytest.fixture(scope="module")
def full(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=VOCAB, seed=32)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    yield s, m
    m.close()


def row(values, vocab):
    """The test's logits followed by -inf (never chosen, weight 0) up to the model's vocabulary."""
    out = np.full(vocab, -np.inf, np.float32)
    out[: len(values)] = values
    return torch.from_numpy(out).cuda()


def mask_of(bits):
    return np.array(bits, bool)


# ---- the reference's unit tests (src/sampling.rs:137-210), through the device ----

def test_impossible_and_corrupt_distributions_are_errors(small):
    smp = qne.Sampler(small)
    with pytest.raises(qne.QneError) as e:
        smp.sample(mask=mask_of([0, 0]), logits=row([1.0, 2.0], 512))
    assert "no finite token is allowed" in str(e.value)
    with pytest.raises(qne.QneError) as e:
        smp.sample(logits=row([math.nan], 512))
    assert "non-finite model logits" in str(e.value)
    with pytest.raises(qne.QneError) as e:
        smp.sample(logits=row([-math.inf], 512))
    assert "no finite token" in str(e.value)


def test_greedy_picks_max_and_respects_mask(small):
    smp = qne.Sampler(small, temperature=0.0)
    lg = row([0.0, 3.0, 1.0, 2.0], 512)
    assert smp.sample(logits=lg) == 1
    assert smp.sample(logits=lg, mask=mask_of([0, 0, 1, 1])) == 3


def test_stochastic_respects_mask_and_top_k(small):
    smp = qne.Sampler(small, temperature=1.0, top_k=1, top_p=1.0, seed=7)
    lg = row([5.0, 4.9, 4.8, -9.0], 512)
    for _ in range(50):
        assert smp.sample(logits=lg, mask=mask_of([0, 1, 0, 1])) == 1


def test_same_seed_is_deterministic_and_matches_the_oracle(small):
    logits = [math.sin(i * 0.7) for i in range(100)]
    lg = row(logits, 512)

    def draw(seed):
        smp = qne.Sampler(small, temperature=1.0, top_k=50, top_p=0.95, seed=seed)
        return [smp.sample(logits=lg) for _ in range(30)]

    def oracle(seed):
        o = OracleSampler(temperature=1.0, top_k=50, top_p=0.95, seed=seed)
        return [o.try_sample(logits) for _ in range(30)]

    assert draw(1) == draw(1)
    assert draw(1) != draw(2)
    assert draw(1) == oracle(1) and draw(2) == oracle(2)


def test_tool_call_bias_flips_greedy(small):
    lg = row([1.0, 3.0, 0.0], 512)
    assert qne.Sampler(small, temperature=0.0).sample(logits=lg) == 1
    assert qne.Sampler(small, temperature=0.0).sample(logits=lg, bias_token=0, bias=4.0) == 0
    assert qne.Sampler(small, temperature=0.0).sample(logits=lg, bias_token=0, bias=-8.0) == 1


def test_presence_penalty_avoids_repeats_but_not_under_a_mask(small):
    lg = row([0.0, 3.0, 2.5, 0.0], 512)
    smp = qne.Sampler(small, temperature=0.0, presence_penalty=1.0)
    assert smp.sample(logits=lg) == 1
    assert smp.sample(logits=lg) == 2
    assert smp.sample(logits=lg, mask=mask_of([0, 1, 1, 0])) == 1


# ---- identical streams on full-vocabulary logits ----

SETTINGS = [
    dict(temperature=0.0),
    dict(temperature=0.6, top_k=20, top_p=0.95, seed=42),
    dict(temperature=1.0, top_k=256, top_p=0.9, seed=3),
    dict(temperature=0.3, top_k=1, top_p=0.95, seed=5),
    dict(temperature=1.5, top_k=100, top_p=1.0, seed=9),
    dict(temperature=0.8, top_k=40, top_p=0.7, seed=11, presence_penalty=1.5),
    dict(temperature=0.0, presence_penalty=2.0),
]


@pytest.mark.parametrize("opts", SETTINGS, ids=[str(i) for i in range(len(SETTINGS))])
@pytest.mark.parametrize("masked", [False, True])
def test_full_vocabulary_streams_match_the_oracle(full, opts, masked):
    _, m = full
    rng = np.random.default_rng(2 * SETTINGS.index(opts) + int(masked))
    smp = qne.Sampler(m, **opts)
    o = OracleSampler(**opts)
    logits_rows = [(rng.standard_normal(VOCAB) * 3).astype(np.float32) for _ in range(4)]
    for step in range(24):
        lg = logits_rows[step % 4]  # repeated rows make the presence penalty matter
        mask = rng.random(VOCAB) < 0.5 if masked else None
        bias_token, bias = (int(rng.integers(0, VOCAB)), 25.0) if step % 7 == 3 else (-1, 0.0)
        got = smp.sample(logits=torch.from_numpy(lg).cuda(), mask=mask, bias_token=bias_token, bias=bias)
        want = o.try_sample(lg, mask=mask, bias_token=bias_token, bias=bias)
        assert got == want, (step, got, want)


def test_failed_draw_leaves_the_generator_unchanged(full):
    _, m = full
    smp = qne.Sampler(m, temperature=1.0, top_k=50, top_p=0.9, seed=77)
    o = OracleSampler(temperature=1.0, top_k=50, top_p=0.9, seed=77)
    lg = (np.random.default_rng(1).standard_normal(VOCAB) * 2).astype(np.float32)
    bad = lg.copy()
    bad[12345] = np.nan
    with pytest.raises(qne.QneError):
        smp.sample(logits=torch.from_numpy(bad).cuda())
    for _ in range(5):
        assert smp.sample(logits=torch.from_numpy(lg).cuda()) == o.try_sample(lg)


def test_step_sample_matches_host_logits_and_greedy_decode(full):
    s, m = full
    prompt = synth.prompt_ids(24, 5, VOCAB)
    # greedy on the device == the engine's fused greedy pick
    m.reset()
    m.prefill(prompt)
    m.snapshot()
    want = m.decode(8, 1)
    m.restore()
    smp = qne.Sampler(m, temperature=0.0)
    tok, pos = m.last_token()
    got = [tok]
    for i in range(7):
        tok = m.step_sample(smp, tok, pos + i)
        got.append(tok)
    assert got == want
    # stochastic: the device draw == the oracle's draw on the host logits of the same step
    opts = dict(temperature=0.7, top_k=30, top_p=0.9, seed=123, presence_penalty=0.5)
    m.restore()
    tok, pos = m.last_token()
    o = OracleSampler(**opts)
    host = []
    t = tok
    for i in range(8):
        t = o.try_sample(m.step(t, pos + i))
        host.append(t)
    m.restore()
    smp = qne.Sampler(m, **opts)
    dev = []
    t = tok
    for i in range(8):
        t = m.step_sample(smp, t, pos + i)
        dev.append(t)
    assert dev == host
