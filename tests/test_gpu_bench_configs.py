"""Parity of the benchmarked paths at the benchmark configurations, against the CPU oracle.

The reference's own parity harness compares whole decodes: 32 greedy tokens, top-1 / top-5 and
logits after the prompt (kernels/src/bin/model_bench.rs:125-153, kernels/src/model.rs:339-372).
Here the engine runs exactly what bench.py times, at the contexts it times:
  config 2  2B f16: the 3968-token prompt through qne_prefill_chunk, then greedy decode on the
            default per-operation path (CUDA graphs of one kernel per operation) to 4000;
  config 3  2B int4 group-64: the 1024-token prompt, then the first 32 of its 256 greedy steps;
  config 4  0.8B f16, 32 sequences with contexts U[256, 4027] on randomly permuted 16-token pages,
            each prompt fed through qne_batch_step: logits after the last prompt token and 16
            greedy steps for 5 sequences, the longest and the shortest among them.
The oracle runs the prompts through its batched CPU path (oracle_model_prefill, checked against
its per-token steps in tests/test_oracle_prefill.py) and the continuations one token at a time.
Logits: max-abs <= 2e-2 and rel_err <= 1e-3. A greedy mismatch passes only at a near-tie (oracle
top-2 margin below 2 x the logit tolerance) and ends the comparison there; the margins of every
compared step are printed (pytest -s) so near-ties are visible."""
import numpy as np
import pytest

import qne
import refchecks as rc
from oracle import oracle
from qne import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
MAX_ABS, REL = 2e-2, 1e-3


def logits_close(got, want, what):
    assert np.all(np.isfinite(got)), what
    err = float(np.abs(got.astype(np.float64) - want).max())
    rel = rc.rel_err(got, want)
    assert err <= MAX_ABS and rel <= REL, (what, err, rel)
    top5_got, top5_want = np.argsort(-got)[:5], np.argsort(-want)[:5]
    return err, rel, len(set(top5_got) & set(top5_want))


def streams_agree(got_ids, want_ids, margins, what):
    """Identical greedy ids, except that a flip at a near-tie ends the comparison. Returns the
    number of identical leading tokens."""
    low = [(i, round(m, 5)) for i, m in enumerate(margins) if m < 2 * MAX_ABS]
    print(f"{what}: min top-2 margin {min(margins):.4g}; near-ties (step, margin) {low}")
    for i, (a, b) in enumerate(zip(got_ids, want_ids)):
        if a != b:
            assert margins[i] < 2 * MAX_ABS, f"{what} token {i}: {a} != {b} with margin {margins[i]}"
            return i
    return len(want_ids)


@pytest.mark.parametrize("cfg,steps", [(2, 32), (3, 32)], ids=["config2-3968", "config3-1024"])
def test_bench_prompt_and_decode_match_the_oracle(cuda, cfg, steps):
    info = synth.baseline_config(cfg)
    s = synth.build_config(cfg)
    m = qne.Model(s.index_json, s.weights)  # the reference architecture loads without opt-in
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    n = info["prompt"]
    prompt = synth.prompt_ids(n, 1 if cfg == 2 else cfg)  # bench.py's prompt for config 2
    m.prefill_chunk(prompt, 0, True)  # bench.py's prompt path
    got = m.logits()
    want = om.prefill_batched(prompt)
    err, rel, top5 = logits_close(got, want, f"config {cfg} after {n} prompt tokens")
    print(f"config {cfg}: logits after the prompt max-abs {err:.3g} rel {rel:.3g}, top-5 overlap {top5}/5")
    m.snapshot()
    om.snapshot()
    want_ids, margins = om.greedy(want, n, steps)
    # every launch path the model offers (the token kernel needs f16 weights), the default first
    paths = [m.path] + [p for p in ("operations", "token") if p != m.path and (p != "token" or cfg == 2)]
    for path in paths:
        m.set_path(path)
        m.restore()
        ids = m.decode(steps, 1)
        same = streams_agree(ids, want_ids, margins, f"config {cfg} greedy ({path})")
        print(f"config {cfg} ({path}): {same}/{steps} greedy tokens identical")
        assert same >= steps // 2
    # per-token logits on each path at the longest contexts
    for path in paths:
        m.set_path(path)
        m.restore()
        om.restore()
        tok = oracle.argmax(want)
        for i in range(4):
            g = m.step(tok, n + i)
            w = om.step(tok, n + i)
            logits_close(g, w, f"config {cfg} step at position {n + i} ({path})")
            tok = oracle.argmax(w)
    m.close()
    om.close()


def test_config4_batched_sequences_match_the_oracle(cuda):
    """32 sequences of the 0.8B f16 model on one weight copy, contexts U[256, 4027] as bench.py
    draws them, permuted page tables; each prompt is fed token by token through qne_batch_step
    (the batched decode kernels the bench times), sequences past their prompt feed back their own
    greedy picks."""
    B, greedy = 32, 16
    s = synth.build_config(4)
    m = qne.Model(s.index_json, s.weights)
    rng = np.random.default_rng(3)
    lens = rng.integers(256, 4027, B, endpoint=True)
    prompts = [synth.prompt_ids(int(lens[b]), 400 + b) for b in range(B)]
    bt = qne.Batch(m, B)
    bt.set_page_table(rng.permutation(B * 256).astype(np.uint32))
    order = np.argsort(lens)
    check = sorted({int(order[-1]), int(order[0]), int(order[B // 2]), int(order[B // 4]), int(order[3 * B // 4])})
    steps_total = int(lens.max()) + greedy
    assert steps_total <= 4096
    tok = np.array([p[0] for p in prompts], np.uint32)
    got_logits, got_ids = {}, {b: [] for b in check}
    for p in range(steps_total - 1):
        want_logits = any(p == lens[b] - 1 for b in check)
        res = bt.step(tok, np.full(B, p, np.uint32), want_logits=want_logits)
        nxt, lg = res if want_logits else (res, None)
        for b in check:
            if p == lens[b] - 1:
                got_logits[b] = lg[b].copy()
            if lens[b] - 1 <= p < lens[b] - 1 + greedy:
                got_ids[b].append(int(nxt[b]))
        tok = np.array([prompts[b][p + 1] if p + 1 < lens[b] else nxt[b] for b in range(B)], np.uint32)
    bt.close()
    m.close()
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    for b in check:
        om.reset()
        want = om.prefill_batched(prompts[b])
        err, rel, top5 = logits_close(got_logits[b], want, f"sequence {b} (context {lens[b]})")
        print(f"config 4 sequence {b}: context {lens[b]}, max-abs {err:.3g} rel {rel:.3g}, top-5 {top5}/5")
        want_ids, margins = om.greedy(want, int(lens[b]), greedy)
        same = streams_agree(got_ids[b], want_ids, margins, f"config 4 sequence {b}")
        print(f"config 4 sequence {b}: {same}/{greedy} greedy tokens identical")
    om.close()
