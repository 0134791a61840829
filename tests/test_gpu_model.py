"""Model-level parity and API semantics on the B200: the whole decode step (CUDA graph of the
sm_100a kernels, either one kernel per operation or one fused launch per layer)
against the CPU oracle on the same random-init weights and token ids.
Logits: max-abs <= 2e-2 and rel_err <= 1e-3; greedy streams identical (steps whose oracle top-2
margin is below the logit tolerance are reported, not failed)."""
import numpy as np
import pytest

import qne
import refchecks as rc
from oracle import oracle
from qne import synth

pytestmark = pytest.mark.gpu
MAX_ABS, REL = 2e-2, 1e-3


def logits_close(got, want):
    assert np.all(np.isfinite(got))
    err = np.abs(got.astype(np.float64) - want).max()
    assert err <= MAX_ABS and rc.rel_err(got, want) <= REL, (err, rc.rel_err(got, want))


def greedy_compare(model, om, prompt, steps):
    """Prefill both, then compare `steps` greedy tokens (GPU-resident loop vs oracle)."""
    model.reset()
    model.prefill(prompt)
    got_logits = model.logits()
    om.reset()
    want_logits = om.prefill(prompt)
    logits_close(got_logits, want_logits)
    ids = model.decode(steps, 1)
    want_ids, margins = om.greedy(want_logits, len(prompt), steps)
    for i, (a, b) in enumerate(zip(ids, want_ids)):
        if a != b:
            assert margins[i] < 2 * MAX_ABS, f"token {i}: {a} != {b} with margin {margins[i]}"
            return i
    return steps


# launches per token: one per operation; one per layer; token kernel launches between the attention
# mixers (every 4th layer here) plus the attention kernels
DISPATCHES = {"operations": lambda layers: 5 * layers + 1, "layers": lambda layers: layers,
              "token": lambda layers: 2 * (layers // 4) + 1}


def set_path(m, path):
    """Launch path: "operations" (one kernel per operation, the default), "layers" (one fused launch
    per layer) or "token" (one launch per token); an error if it is not available (f16 weights on a
    B200 for the last two)."""
    m.set_path(path)
    assert m.path == path and m.fused == (path == "layers")
    assert m.dispatches_per_token() == DISPATCHES[path](m.layers)


@pytest.fixture(scope="module", params=[("f16", "layers"), ("f16", "operations"), ("f16", "token"),
                                        ("q4g64", "operations"), ("q4", "operations")],
                ids=["f16-fused", "f16-split", "f16-token", "q4g64", "q4"])
def tiny(request, cuda):
    kind, fused = request.param
    s = synth.build(1024, 3584, layers=4, vocab=8192, kind=kind, seed=11)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    set_path(m, fused)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    yield kind, s, m, om
    m.close()
    om.close()


def test_tiny_model_prefill_and_greedy(tiny):
    kind, s, m, om = tiny
    prompt = synth.prompt_ids(40, 0, 8192)
    n = greedy_compare(m, om, prompt, 32)
    assert n == 32


def test_step_matches_oracle_and_leaves_the_pick(tiny):
    kind, s, m, om = tiny
    prompt = synth.prompt_ids(10, 1, 8192)
    m.reset()
    m.prefill(prompt)
    pick, pos = m.last_token()
    om.reset()
    want = om.prefill(prompt)
    assert (pick, pos) == (oracle.argmax(want), 10)
    lg = m.step(1234, 10)
    logits_close(lg, om.step(1234, 10))
    assert m.last_token() == (1234, 10)  # step writes (token, pos) and skips the greedy pick
    lg2 = m.step(77, 11)
    logits_close(lg2, om.step(77, 11))


def test_snapshot_restore_and_reset_are_exact(tiny):
    kind, s, m, om = tiny
    prompt = synth.prompt_ids(12, 2, 8192)
    m.reset()
    m.prefill(prompt)
    m.snapshot()
    a = m.step(5, 12).copy()
    m.step(6, 13)
    m.restore()
    assert m.last_token() == (m.last_token()[0], 12)
    b = m.step(5, 12)
    assert np.array_equal(a, b)
    m.reset()
    m.prefill(prompt)
    c = m.step(5, 12)
    assert np.array_equal(a, c)


def test_chunked_prefill_equals_one_pass(tiny):
    kind, s, m, om = tiny
    prompt = synth.prompt_ids(50, 3, 8192)
    m.reset()
    m.prefill(prompt)
    a = m.logits().copy()
    m.reset()
    m.prefill_chunk(prompt[:32], 0, False)
    m.prefill_chunk(prompt[32:], 32, True)
    # batched chunks (tensor-core GEMMs; int4 matrices decoded to f16 first): within the tolerance
    logits_close(m.logits(), a.astype(np.float64))
    assert m.last_token()[1] == 50


def test_decode_windows_and_stops(tiny):
    kind, s, m, om = tiny
    prompt = synth.prompt_ids(8, 4, 8192)
    m.reset()
    m.prefill(prompt)
    m.snapshot()
    one = m.decode(9, 1)
    m.restore()
    win = m.decode(9, 4)
    assert win[0] == one[0] and win[1:5] == [0xFFFFFFFF] * 4
    m.restore()
    stop_at = next((i for i, t in enumerate(one) if t != one[0]), None)
    stop_tok = one[stop_at] if stop_at is not None else one[0]
    want = one[: (stop_at if stop_at is not None else 0) + 1]
    stopped = m.decode(9, 1, stop=[stop_tok])
    assert stopped == want
    m.restore()
    m.decode(5, 4)
    assert m.last_token() == (one[4], 8 + 4)


def test_context_limits_and_errors(tiny):
    kind, s, m, om = tiny
    with pytest.raises(qne.QneError) as e:
        m.prefill_chunk([1, 2, 3], 4094, True)
    assert e.value.name == "ERANGE_CTX"
    with pytest.raises(qne.QneError) as e:
        m.step(1, 4096)
    assert e.value.name == "ERANGE_CTX"
    with pytest.raises(qne.QneError) as e:
        m.prefill(np.zeros(4096, np.uint32))
    assert e.value.name == "ERANGE_CTX"
    m.reset()
    m.prefill(synth.prompt_ids(4, 5, 8192))
    with pytest.raises(qne.QneError) as e:
        m.decode(5000, 64)  # fails before a window would run past position 4095
    assert e.value.name == "ERANGE_CTX"
    assert m.last_token()[1] <= 4096


def test_restore_without_snapshot(cuda):
    s = synth.build(1024, 3584, layers=4, vocab=512, seed=12)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    with pytest.raises(qne.QneError) as e:
        m.restore()
    assert e.value.name == "ENOSNAP"
    assert not m.fused and m.dispatches_per_token() == 4 * 5 + 1  # per-operation path by default
    m.set_fused(True)
    assert m.dispatches_per_token() == 4  # one fused launch per layer
    m.set_path("token")
    assert m.dispatches_per_token() == 3 and not m.fused  # token kernel, attention, token kernel
    assert "B200" in m.adapter or "sm_10" in m.adapter
    m.close()


def test_launch_paths_agree(cuda):
    """The three launch paths on one model: logits within the parity tolerance, identical picks,
    and switching paths mid-sequence keeps the state (all read and write the same buffers)."""
    s = synth.build(1024, 3584, layers=8, vocab=8192, seed=13)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    prompt = synth.prompt_ids(70, 6, 8192)
    out = {}
    for path in ("layers", "operations", "token"):
        set_path(m, path)
        m.reset()
        m.prefill(prompt)
        out[path] = (m.logits().copy(), m.decode(12, 1))
    for path in ("layers", "token"):
        logits_close(out[path][0], out["operations"][0].astype(np.float64))
        assert out[path][1] == out["operations"][1]
    m.set_fused(True)
    m.reset()
    m.prefill(prompt[:40])
    m.set_path("token")
    for i in range(40, 55):  # one token per step on the token kernel (Model::step)
        m.step(int(prompt[i]), i)
    m.set_fused(False)
    m.prefill_chunk(prompt[55:], 55, True)
    logits_close(m.logits(), out["operations"][0].astype(np.float64))
    m.close()


def test_fused_kernels_at_a_long_context(cuda):
    """Attention splits of the fused kernel past one 64-token block and past 8 groups of splits:
    prefill 600 tokens, then compare against the per-operation kernels."""
    s = synth.build(1024, 3584, layers=4, vocab=4096, seed=14)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    prompt = synth.prompt_ids(600, 7, 4096)
    res = []
    for path in ("layers", "token", "operations"):
        set_path(m, path)
        m.reset()
        m.prefill(prompt)
        res.append((m.logits().copy(), m.decode(6, 1)))
    for r in res[:2]:
        logits_close(r[0], res[2][0].astype(np.float64))
        assert r[1] == res[2][1]
    m.close()


@pytest.mark.slow
@pytest.mark.parametrize("fused", ["layers", "operations", "token"], ids=["fused", "split", "token"])
def test_config1_full_08b_parity(cuda, fused):
    """benchmark config 1: 0.8B-shaped f16 model (seed 0), 128 prompt ids (seed 0), greedy steps."""
    s = synth.build_config(1)
    m = qne.Model(s.index_json, s.weights)
    set_path(m, fused)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    prompt = synth.prompt_ids(128, 0)
    n = greedy_compare(m, om, prompt, 32)
    assert n == 32
    m.close()
    om.close()


@pytest.mark.slow
@pytest.mark.parametrize("cfg,fused", [(2, "operations"), (2, "layers"), (2, "token"), (3, "operations")],
                         ids=["config2-split", "config2-fused", "config2-token", "config3"])
def test_config_2b_short_context_parity(cuda, cfg, fused):
    """benchmark configs 2 (f16, both launch paths) and 3 (int4 g64) from a short prompt, one token
    per step (qne_prefill); the benchmark contexts themselves are in test_gpu_bench_configs.py."""
    s = synth.build_config(cfg)
    m = qne.Model(s.index_json, s.weights)
    set_path(m, fused)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    prompt = synth.prompt_ids(48, cfg)
    n = greedy_compare(m, om, prompt, 32)
    assert n == 32
    m.close()
    om.close()


def test_sync_deadline_reports_a_timeout(cuda):
    """qne_sync / qne_batch_sync poll the stream with a deadline (the reference's GPU wait,
    kernels/src/lib.rs:398-405, fails with an error instead of hanging). The stream is held by a
    bounded spin kernel (torch.cuda._sleep, about one second) so that a 1 ms deadline runs out."""
    import torch
    s = synth.build(1024, 3584, layers=4, vocab=4096, seed=16)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    st = torch.cuda.Stream()
    m.set_stream(st.cuda_stream)
    bt = qne.Batch(m, 2)
    for hold in (lambda: m.sync(1), lambda: bt.sync(1)):
        with torch.cuda.stream(st):
            torch.cuda._sleep(2_000_000_000)
        with pytest.raises(qne.QneError) as e:
            hold()
        assert e.value.name == "ETIMEOUT" and "exceeded" in str(e.value)
        m.sync()  # the spin ends; a normal wait succeeds
    m.prefill(synth.prompt_ids(5, 1, 4096))
    assert m.last_token()[1] == 5
    bt.close()
    m.close()


@pytest.mark.parametrize("path", ["layers", "token"])
def test_barrier_wait_runs_out_and_reports_a_timeout(cuda, path):
    """The grid barriers of the fused layer kernels and of the token kernel are bounded waits. With
    the test hook every barrier also waits for an arrival that never comes, under a 1 ms limit: the
    kernels set the timeout flag and return (no hang, the context stays usable), qne_last_token
    reports QNE_ETIMEOUT and clears the flag, and with the hook off the same prompt gives the same
    bits as before."""
    import time
    s = synth.build(1024, 3584, layers=4, vocab=4096, seed=15)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    set_path(m, path)
    prompt = synth.prompt_ids(9, 2, 4096)
    m.prefill(prompt)
    want, want_ids = m.logits().copy(), m.decode(4, 1)
    m.test_barrier_timeout(1000)
    m.reset()
    t0 = time.perf_counter()
    m.prefill(prompt[:3])
    with pytest.raises(qne.QneError) as e:
        m.last_token()
    assert e.value.name == "ETIMEOUT" and "timed out" in str(e.value)
    assert time.perf_counter() - t0 < 5.0  # one limit, not one per barrier
    m.test_barrier_timeout(0)
    m.reset()
    m.prefill(prompt)
    assert np.array_equal(m.logits(), want) and m.decode(4, 1) == want_ids
    m.close()


def test_profile_token_times_every_dispatch_and_consumes_one_token(cuda):
    """Model::profile_token (kernels/src/model.rs:305-307): one greedy token, milliseconds per
    dispatch label; afterwards the model stands where one decode step leaves it."""
    s = synth.build(1024, 3584, layers=4, vocab=4096, seed=17)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    m.prefill(synth.prompt_ids(20, 3, 4096))
    m.snapshot()
    want = m.decode(2, 1)
    m.restore()
    prof = m.profile_token()
    assert set(prof) == {"gemv_8224x1024_Store", "gemv_5120x1024_Store", "gemv_1024x2048_Accumulate",
                         "gemv_7168x1024_SwiGlu", "gemv_1024x3584_Accumulate", "gemv_4096x1024_Argmax", "gdn",
                         "attention"}, prof
    assert all(0.0 < v < 50.0 for v in prof.values()), prof
    assert m.last_token() == (want[1], 21)
    m.close()


def test_dispatch_cost_probe(cuda):
    """The reference's dispatch-cost probe (noop kernel, kernels/src/lib.rs:718-724) in the four
    launch modes: every launch runs (y counts them) and costs a few microseconds at most."""
    import torch
    y = torch.zeros(1, device="cuda")
    n, total = 500, 0
    for mode, warm in (("plain", 10), ("graph", n), ("pdl", 10), ("graph_pdl", n)):
        us = qne.dispatch_cost(n, mode, y)
        total += n + warm
        torch.cuda.synchronize()
        assert 0.0 < us < 20.0, (mode, us)
        assert int(y.item()) == total, mode
        print(f"dispatch cost {mode}: {us:.2f} us per launch")
