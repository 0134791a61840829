"""The CPU restatement of the reference sampler (oracle/sampler.py) against the reference's own
unit tests (src/sampling.rs:137-210, same inputs and expectations), plus its generator: the
checker the device sampler is compared with."""
import math

import numpy as np
import pytest

from oracle.sampler import Sampler


def greedy(**kw):
    return Sampler(temperature=0.0, **kw)


def test_impossible_and_corrupt_distributions_are_errors():
    s = Sampler()
    with pytest.raises(ValueError):
        s.try_sample([1.0, 2.0], mask=np.zeros(2, bool))
    with pytest.raises(ValueError):
        s.try_sample([math.nan])
    with pytest.raises(ValueError):
        s.try_sample([-math.inf])
    with pytest.raises(ValueError):
        s.try_sample([])


def test_greedy_picks_max_and_respects_mask():
    logits = [0.0, 3.0, 1.0, 2.0]
    s = greedy()
    assert s.try_sample(logits) == 1
    assert s.try_sample(logits, mask=np.array([0, 0, 1, 1], bool)) == 3


def test_stochastic_respects_mask_and_top_k():
    logits = [5.0, 4.9, 4.8, -9.0]
    mask = np.array([0, 1, 0, 1], bool)
    s = Sampler(temperature=1.0, top_k=1, top_p=1.0, seed=7)
    for _ in range(50):
        assert s.try_sample(logits, mask=mask) == 1


def test_same_seed_is_deterministic():
    logits = [math.sin(i * 0.7) for i in range(100)]

    def draw(seed):
        s = Sampler(temperature=1.0, top_k=50, top_p=0.95, seed=seed)
        return [s.try_sample(logits) for _ in range(30)]

    assert draw(1) == draw(1)
    assert draw(1) != draw(2)


def test_tool_call_bias_flips_greedy():
    logits = [1.0, 3.0, 0.0]
    assert greedy().try_sample(logits) == 1
    assert greedy().try_sample(logits, bias_token=0, bias=4.0) == 0
    assert greedy().try_sample(logits, bias_token=0, bias=-8.0) == 1


def test_presence_penalty_avoids_repeats_but_not_under_a_mask():
    logits = [0.0, 3.0, 2.5, 0.0]
    s = greedy(presence_penalty=1.0)
    assert s.try_sample(logits) == 1
    assert s.try_sample(logits) == 2, "token 1 is penalised once generated"
    assert s.try_sample(logits, mask=np.array([0, 1, 1, 0], bool)) == 1, "no penalty inside the grammar"


def test_generator_matches_the_reference_formula():
    # state = seed * 0x9E3779B97F4A7C15 | 1; xorshift (13, 7, 17); (x >> 40) / 2^24
    s = Sampler(seed=42)
    x = (42 * 0x9E3779B97F4A7C15) & ((1 << 64) - 1) | 1
    for _ in range(5):
        x ^= (x << 13) & ((1 << 64) - 1)
        x ^= x >> 7
        x ^= (x << 17) & ((1 << 64) - 1)
        assert s.next_f32() == np.float32(x >> 40) / np.float32(1 << 24)
