"""Batched prompt processing (qne_prefill_chunk: 64-token chunks through the
tensor-core GEMMs, the chunked GDN scan, K/V append + causal attention) against the CPU oracle
and against the per-token path (qne_prefill), on the same random-init weights and token ids.

Logits: max-abs <= 2e-2 and rel_err <= 1e-3 after the prompt AND after decode steps that read
the state the chunk left (GDN recurrent state, conv ring, KV pages); greedy picks identical
(picks whose oracle top-2 margin is below the logit tolerance are reported, not failed)."""
import numpy as np
import pytest

import qne
import refchecks as rc
from oracle import oracle
from qne import synth

pytestmark = pytest.mark.gpu
MAX_ABS, REL = 2e-2, 1e-3
VOCAB = 8192


def logits_close(got, want):
    assert np.all(np.isfinite(got))
    err = np.abs(got.astype(np.float64) - want).max()
    assert err <= MAX_ABS and rc.rel_err(got, want) <= REL, (err, rc.rel_err(got, want))


def same_pick(got_logits, want_logits):
    a, b = oracle.argmax(got_logits), oracle.argmax(want_logits)
    if a != b:
        top2 = np.partition(want_logits, -2)[-2:]
        assert abs(top2[1] - top2[0]) < 2 * MAX_ABS, (a, b)


@pytest.fixture(scope="module")
def tiny(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="f16", seed=21)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    yield m, om
    m.close()
    om.close()


def steps_after(m, om, tokens, pos):
    """Host-token steps after a prefill: each step's logits must match the oracle's."""
    for i, t in enumerate(tokens):
        logits_close(m.step(int(t), pos + i), om.step(int(t), pos + i))


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 31, 32, 33, 63, 64, 65, 100, 130])
def test_batched_prefill_matches_oracle(tiny, n):
    """Ragged chunk sizes (1..64 rows, several chunks): logits, the greedy pick left in the
    control words, and the state the decode steps read afterwards."""
    m, om = tiny
    prompt = synth.prompt_ids(n, 100 + n, VOCAB)
    m.reset()
    m.prefill_chunk(prompt, 0, True)  # the first call of a chunk size also records its graph
    launches0 = qne.kernel_launches()
    m.reset()
    m.prefill_chunk(prompt, 0, True)
    launched = qne.kernel_launches() - launches0
    chunks = -(-n // qne.PREFILL_CHUNK_TOKENS)
    # embedding prep + per layer (GEMM, mixer, 3 GEMMs; + the gated-norm prep for GDN layers, + kv_append
    # for attention layers, whose merge writes the out-projection's planes itself) + chunk finish
    per_chunk = 6 * m.layers + 2
    assert launched == chunks * per_chunk + 1  # + the LM head
    if n > 2:
        assert launched < n * m.dispatches_per_token()  # the weights stream once per chunk
    got = m.logits()
    om.reset()
    want = om.prefill(prompt)
    logits_close(got, want)
    tok, pos = m.last_token()
    assert pos == n
    same_pick(got, want)
    if tok != oracle.argmax(want):
        return  # a near-tie picked the other token; the state checks below would diverge
    steps_after(m, om, synth.prompt_ids(6, 200 + n, VOCAB), n)


def test_non_finish_chunks_then_finish(tiny):
    """prefill_chunk(finish=False) leaves (last id, its position) and skips the LM head; the next
    chunk continues the same state."""
    m, om = tiny
    prompt = synth.prompt_ids(77, 7, VOCAB)
    m.reset()
    m.prefill_chunk(prompt[:20], 0, False)
    assert m.last_token() == (int(prompt[19]), 19)
    m.prefill_chunk(prompt[20:45], 20, False)
    assert m.last_token() == (int(prompt[44]), 44)
    m.prefill_chunk(prompt[45:], 45, True)
    om.reset()
    want = om.prefill(prompt)
    logits_close(m.logits(), want)
    assert m.last_token()[1] == 77
    ids = m.decode(12, 1)
    want_ids, margins = om.greedy(want, 77, 12)
    for i, (a, b) in enumerate(zip(ids, want_ids)):
        if a != b:
            assert margins[i] < 2 * MAX_ABS, (i, a, b)
            break


def test_mixing_per_token_and_batched_prefill(tiny):
    """A per-token prefill, then a batched chunk that continues it, then host steps: the two paths
    share the conv ring (slot = token index % 4), the recurrent states and the KV pages."""
    m, om = tiny
    prompt = synth.prompt_ids(59, 8, VOCAB)
    for split in (1, 2, 3, 6, 37):
        m.reset()
        m.prefill(prompt[:split])
        m.prefill_chunk(prompt[split:], split, True)
        om.reset()
        want = om.prefill(prompt)
        logits_close(m.logits(), want)
    steps_after(m, om, synth.prompt_ids(4, 9, VOCAB), 59)
    # and the other way round: batched first, then per-token steps through the same state
    m.reset()
    m.prefill_chunk(prompt[:45], 0, False)
    om.reset()
    om.prefill(prompt[:45])
    steps_after(m, om, prompt[45:], 45)


def test_batched_prefill_after_snapshot_restore(tiny):
    m, om = tiny
    prompt = synth.prompt_ids(40, 10, VOCAB)
    m.reset()
    m.prefill_chunk(prompt[:30], 0, True)
    m.snapshot()
    m.prefill_chunk(prompt[30:], 30, True)
    a = m.logits().copy()
    m.restore()
    m.prefill_chunk(prompt[30:], 30, True)
    assert np.array_equal(a, m.logits())  # the same kernels on the same state: bitwise equal


def test_batched_prefill_long_context_agrees_with_per_token(cuda):
    """600 tokens: attention over many 256-token splits and merge groups per row; batched and
    per-token prefill give logits within the tolerance and the same greedy continuation."""
    s = synth.build(1024, 3584, layers=4, vocab=4096, seed=22)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    prompt = synth.prompt_ids(600, 11, 4096)
    m.prefill(prompt)
    a, ids_a = m.logits().copy(), m.decode(8, 1)
    m.reset()
    m.prefill_chunk(prompt, 0, True)
    b, ids_b = m.logits().copy(), m.decode(8, 1)
    logits_close(b, a.astype(np.float64))
    assert ids_a == ids_b
    m.close()


@pytest.mark.parametrize("kind", ["q4", "q4g64"])
@pytest.mark.parametrize("n", [20, 64, 100])
def test_int4_batched_prefill(cuda, kind, n):
    """int4 decoder matrices (the reference converter's block-32 layout, and group 64): the chunk
    GEMMs widen the nibbles to f16 in shared memory (no decode launches). Logits against the
    oracle and against the per-token path (qne_prefill), the greedy continuation, and the launch
    count."""
    s = synth.build(1024, 3584, layers=4, vocab=4096, kind=kind, embed_kind="q4" if kind == "q4" else "f16",
                    seed=23)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    assert m.prefill_batched_supported
    prompt = synth.prompt_ids(n, 12, 4096)
    m.prefill(prompt)
    a, ids_a = m.logits().copy(), m.decode(8, 1)
    m.reset()
    m.prefill_chunk(prompt, 0, True)  # records the chunk graphs
    m.reset()
    launches0 = qne.kernel_launches()
    m.prefill_chunk(prompt, 0, True)
    per_chunk = 6 * m.layers + 2  # as for f16 weights
    assert qne.kernel_launches() - launches0 == -(-n // qne.PREFILL_CHUNK_TOKENS) * per_chunk + 1
    b = m.logits().copy()
    want = om.prefill(prompt)
    logits_close(b, want)
    logits_close(b, a.astype(np.float64))
    same_pick(b, want)
    ids_b = m.decode(8, 1)
    want_ids, margins = om.greedy(want, n, 8)
    for i, (x, y) in enumerate(zip(ids_b, want_ids)):
        if x != y:
            assert margins[i] < 2 * MAX_ABS, (i, x, y)
            break
    if ids_a != ids_b:  # per-token and batched agree unless a near-tie flipped a pick
        i = next(i for i, (x, y) in enumerate(zip(ids_a, ids_b)) if x != y)
        assert margins[i] < 2 * MAX_ABS
    m.close()
    om.close()


@pytest.mark.slow
def test_config2_batched_prefill_of_the_bench_prompt(cuda):
    """benchmark config 2 (2B f16): the bench's 3968-token prompt through the batched path and
    through the per-token path: logits within the tolerance, 32 identical greedy tokens."""
    s = synth.build_config(2)
    m = qne.Model(s.index_json, s.weights)
    prompt = synth.prompt_ids(3968, 1)
    m.prefill(prompt)
    a, ids_a = m.logits().copy(), m.decode(32, 1)
    m.reset()
    m.prefill_chunk(prompt, 0, True)
    b, ids_b = m.logits().copy(), m.decode(32, 1)
    logits_close(b, a.astype(np.float64))
    assert ids_a == ids_b
    m.close()
