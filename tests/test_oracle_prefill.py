"""The oracle's batched prompt path (oracle_model_prefill: all tokens of each matrix product at
once, the GDN recurrence and causal attention over the whole run) against n per-token oracle steps
on the same synthetic model. It is the checker of the GPU tests at the benchmark contexts (3968
tokens), so it is itself checked here: the same logits and states within f32 reordering of the
matrix products, the same greedy continuation."""
import numpy as np
import pytest

import refchecks as rc
from oracle import oracle
from qne import synth

TOL = 2e-5  # relative: only the f32 summation order of the matrix products differs


@pytest.mark.parametrize("kind", ["f16", "q4", "q4g64"])
@pytest.mark.parametrize("epilogue", [0, 1, 2])
def test_gemm_tokens_matches_gemv_per_token(kind, epilogue):
    rng = np.random.default_rng(5 + epilogue)
    rows, k, n = 40, 320, 7
    el = rows * k
    if kind == "f16":
        w, s, z = (rng.standard_normal(el) * 0.05).astype(np.float16), None, None
    else:
        w = rng.integers(0, 2**32, el // 8, dtype=np.uint64).astype(np.uint32)
        if kind == "q4":
            s = np.abs(rng.standard_normal(el // 32) * 0.01).astype(np.float16)
            z = np.full(el // 256, 0x76543210, np.uint32)
        else:
            s = np.abs(rng.standard_normal(el // 64) * 0.01).astype(np.float16)
            z = np.full(el // 64, 7.5, np.float16)
    out = rows // 2 if epilogue == 2 else rows
    x = rng.standard_normal((n, k)).astype(np.float32)
    y0 = rng.standard_normal((n, out)).astype(np.float32)
    got = oracle.gemm_tokens(kind, w, s, z, rows, k, x, y0.copy(), epilogue)
    for t in range(n):
        want = oracle.gemv(kind, w, s, z, rows, k, x[t], y0[t].copy(), epilogue)
        assert rc.rel_err(got[t], want) <= TOL


@pytest.fixture(scope="module")
def small():
    return synth.build(1024, 3584, layers=8, vocab=4096, kind="f16", seed=61)


def test_batched_prefill_matches_per_token_steps(small):
    prompt = synth.prompt_ids(150, 3, 4096)
    a = oracle.OracleModel(small.index_json, small.weights, kv_f16=True)
    b = oracle.OracleModel(small.index_json, small.weights, kv_f16=True)
    want = a.prefill(prompt)
    got = b.prefill_batched(prompt)
    assert rc.rel_err(got, want) <= TOL
    for layer in (0, 3, 6):  # GDN state + conv window, attention K/V (f16), GDN again
        wa, wb = a.state(layer, len(prompt))
        ga, gb = b.state(layer, len(prompt))
        # f16 keys/values: a reordered sum can move a value across an f16 rounding boundary (one
        # f16 step is 2^-11 relative)
        tol = 1e-3 if (layer + 1) % 4 == 0 else 1e-4
        assert rc.rel_err(ga, wa) <= tol and rc.rel_err(gb, wb) <= tol
    # the continuation from either state picks the same tokens
    ids_a, _ = a.greedy(want, len(prompt), 8)
    ids_b, _ = b.greedy(got, len(prompt), 8)
    assert ids_a == ids_b
    a.close()
    b.close()


def test_batched_prefill_continues_a_per_token_prefix_and_restores(small):
    prompt = synth.prompt_ids(90, 4, 4096)
    a = oracle.OracleModel(small.index_json, small.weights, kv_f16=True)
    b = oracle.OracleModel(small.index_json, small.weights, kv_f16=True)
    want = a.prefill(prompt)
    b.prefill(prompt[:31])
    b.snapshot()
    got = b.prefill_batched(prompt[31:], 31)
    assert rc.rel_err(got, want) <= TOL
    b.restore()  # back to 31 tokens: the same chunk again gives the same bits
    assert np.array_equal(b.prefill_batched(prompt[31:], 31), got)
    with pytest.raises(ValueError):
        b.prefill_batched([1, 2, 3], 4094)
    a.close()
    b.close()
