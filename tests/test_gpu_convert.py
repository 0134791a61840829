"""Converted weight files on the B200: a q4 model (the reference converter's layout) and its
f16 conversion, and an f16 model and its q4g64 conversion, each loaded through qne_model_load and
compared with the CPU oracle on the same file (logits max-abs <= 2e-2, rel <= 1e-3, greedy picks);
the batched prefill path over the f16 conversion."""
import numpy as np
import pytest

import qne
import refchecks as rc
from oracle import oracle
from qne import convert, synth

pytestmark = pytest.mark.gpu
VOCAB = 4096


def check(index_json, weights, prompt):
    m = qne.Model(index_json, weights, any_shape=True)
    om = oracle.OracleModel(index_json, weights, kv_f16=True)
    m.prefill(prompt)
    got, want = m.logits(), om.prefill(prompt)
    err = np.abs(got.astype(np.float64) - want).max()
    assert err <= 2e-2 and rc.rel_err(got, want) <= 1e-3, err
    ids, (want_ids, margins) = m.decode(8, 1), om.greedy(want, len(prompt), 8)
    for i, (a, b) in enumerate(zip(ids, want_ids)):
        if a != b:
            assert margins[i] < 4e-2, (i, a, b)
            break
    return m, om, got


def test_q4_source_and_its_f16_conversion(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="q4", embed_kind="q4", seed=51)
    prompt = synth.prompt_ids(20, 3, VOCAB)
    m0, om0, l0 = check(s.index_json, s.weights, prompt)
    assert m0.prefill_batched_supported  # int4 chunks decode each matrix to f16 first
    idx, w = convert.convert(s.index_json, s.weights, "f16")
    m1, om1, l1 = check(idx, w, prompt)
    assert m1.prefill_batched_supported
    m1.reset()
    m1.prefill_chunk(prompt, 0, True)  # the batched path over the converted file
    lb = m1.logits()
    assert np.abs(lb.astype(np.float64) - l1).max() <= 2e-2
    assert np.abs(l1.astype(np.float64) - l0).max() <= 2e-2 * max(1.0, float(np.abs(l0).max()))
    for x in (m0, om0, m1, om1):
        x.close()


def test_f16_source_and_its_q4g64_conversion(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=VOCAB, kind="f16", seed=52)
    idx, w = convert.convert(s.index_json, s.weights, "q4g64", embed_kind="f16")
    m, om, _ = check(idx, w, synth.prompt_ids(16, 4, VOCAB))
    m.close()
    om.close()
